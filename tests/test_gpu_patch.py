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
