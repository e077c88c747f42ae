"""FP8 model patching on the GPU: a random-init HF Whisper encoder (large-v3 widths, 2 layers)
with every encoder linear replaced by the FP8 GEMM (fp8_e4m3 preset) and every LayerNorm by the
fused kernel.

Gates: each patched linear, fed its own captured input, matches the fp32 oracle GEMM of the same
quantised operands (max relative error <= 1e-2); the patched encoder output tracks the unpatched
fp16 encoder statistically (cosine >= 0.99): per-tensor FP8 rounding of every linear is the only
intended difference.
"""
import pytest
import torch
import torch.nn.functional as F

from oracle import fp8, gemm

pytestmark = pytest.mark.gpu


def _encoder(dev):
    from transformers import WhisperConfig
    from transformers.models.whisper.modeling_whisper import WhisperEncoder
    torch.manual_seed(0)
    cfg = WhisperConfig(d_model=1280, encoder_layers=2, encoder_attention_heads=20, encoder_ffn_dim=5120,
                        num_mel_bins=128, max_source_positions=1500, pad_token_id=0, bos_token_id=1,
                        eos_token_id=2, decoder_start_token_id=1)
    enc = WhisperEncoder(cfg).eval()
    with torch.no_grad():
        for name, p in enc.named_parameters():
            if name.endswith("weight") and p.dim() == 2:
                p.normal_(0.0, 0.02)
    return enc.half().to(dev)


def test_patched_encoder_fp8(cuda_device):
    from whisper_blaze_b200.modules import BlazeLinear
    from whisper_blaze_b200.patch import patch_layers
    from whisper_blaze_b200.precision import fp8_e4m3
    enc = _encoder(cuda_device)
    feats = torch.randn(2, 128, 3000, generator=torch.Generator().manual_seed(1)).half().to(cuda_device)
    with torch.no_grad():
        ref = enc(feats).last_hidden_state.float()
    counts = patch_layers(enc, fp8_e4m3())
    assert counts["patched_linears"] == 12 and counts["patched_layernorms"] == 5
    assert counts["fp8_encoder_attn_qkv"] == 6 and counts["fp8_encoder_ffn"] == 4
    seen = {}

    def hook(name):
        def fn(mod, inp, out):
            seen[name] = (mod, inp[0].detach().clone(), out.detach().clone())
        return fn

    for name in ("layers.0.self_attn.q_proj", "layers.0.fc1", "layers.1.fc2"):
        mod = enc.get_submodule(name)
        assert isinstance(mod, BlazeLinear)
        mod.register_forward_hook(hook(name))
    with torch.no_grad():
        out = enc(feats).last_hidden_state.float()
    assert torch.isfinite(out).all()
    cos = F.cosine_similarity(out.view(-1), ref.view(-1), dim=0).item()
    assert cos >= 0.99, f"cosine vs fp16 encoder {cos:.5f}"
    for name, (mod, x, y) in seen.items():
        xq, sx = fp8.quantise(x.reshape(-1, x.shape[-1]).cpu().numpy(), fp8.E4M3)
        ref32 = gemm.gemm_fp8_ref_f32(torch.from_numpy(xq), float(sx), mod._w_fp8.cpu(), float(mod._w_scale.item()),
                                      None if mod._bias16 is None else mod._bias16.cpu())
        rel = gemm.rel_error(y.reshape(-1, y.shape[-1]).float().cpu(), ref32)
        assert rel <= 1e-2, f"{name}: max relative error {rel:.3e}"


def test_patched_decoder_stacked_cross_kv(cuda_device):
    """Decoder layers (large-v3 widths, 2 layers): encoder_attn.k_proj / v_proj run as ONE stacked
    FP8 GEMM [2560, 1280] per layer and forward (one per-tensor weight scale, config 4's shape);
    its output matches the fp32 oracle of the same quantised operands; the patched decoder tracks
    the fp16 decoder (cosine >= 0.99)."""
    from transformers import WhisperConfig
    from transformers.models.whisper.modeling_whisper import WhisperDecoder
    from whisper_blaze_b200.patch import patch_layers
    from whisper_blaze_b200.precision import fp8_e4m3
    torch.manual_seed(0)
    cfg = WhisperConfig(d_model=1280, decoder_layers=2, decoder_attention_heads=20, decoder_ffn_dim=5120,
                        vocab_size=51866, max_target_positions=448, pad_token_id=0, bos_token_id=1,
                        eos_token_id=2, decoder_start_token_id=1)
    dec = WhisperDecoder(cfg).eval()
    with torch.no_grad():
        for name, p in dec.named_parameters():
            if name.endswith("weight") and p.dim() == 2:
                p.normal_(0.0, 0.02)
    dec = dec.half().to(cuda_device)
    g = torch.Generator().manual_seed(3)
    ids = torch.randint(3, 51866, (2, 4), generator=g).to(cuda_device)
    states = torch.randn(2, 1500, 1280, generator=g).half().to(cuda_device)
    with torch.no_grad():
        ref = dec(input_ids=ids, encoder_hidden_states=states, use_cache=False).last_hidden_state.float()
    counts = patch_layers(dec, fp8_e4m3())
    assert counts["stacked_cross_kv"] == 2 and counts["patched_linears"] == 2 * 10
    kv = dec.layers[0].encoder_attn.kv_proj
    seen = []
    kv.linear.register_forward_hook(lambda mod, inp, out: seen.append((inp[0].detach().clone(), out.detach().clone())))
    with torch.no_grad():
        out = dec(input_ids=ids, encoder_hidden_states=states, use_cache=False).last_hidden_state.float()
    assert len(seen) == 1, "the stacked K/V GEMM must run once per layer and forward"
    assert torch.isfinite(out).all()
    cos = F.cosine_similarity(out.view(-1), ref.view(-1), dim=0).item()
    assert cos >= 0.99, f"cosine vs fp16 decoder {cos:.5f}"
    x, y = seen[0]
    assert y.shape[-1] == 2560
    xq, sx = fp8.quantise(x.reshape(-1, 1280).cpu().numpy(), fp8.E4M3)
    ref32 = gemm.gemm_fp8_ref_f32(torch.from_numpy(xq), float(sx), kv.linear._w_fp8.cpu(),
                                  float(kv.linear._w_scale.item()), kv.linear._bias16.cpu())
    rel = gemm.rel_error(y.reshape(-1, 2560).float().cpu(), ref32)
    assert rel <= 1e-2, f"stacked K/V: max relative error {rel:.3e}"
