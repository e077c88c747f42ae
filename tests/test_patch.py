"""Model patching (the reference's WhisperBlaze._patch_layers, whisper_blaze/model.py:334-350,
extended to the FP8 linears of each PrecisionConfig group) on a tiny random-init HF Whisper
model on the CPU: module selection per group, and bit-identical outputs for the fp16 preset
(BlazeLinear's fp16 branch is F.linear; BlazeLayerNorm falls back to F.layer_norm off the GPU)."""
import pytest
import torch

from whisper_blaze_b200.modules import BlazeLayerNorm, BlazeLinear
from whisper_blaze_b200.patch import linear_group, patch_layers
from whisper_blaze_b200.precision import full_fp16


def _tiny_model():
    from transformers import WhisperConfig
    from transformers.models.whisper.modeling_whisper import WhisperModel
    torch.manual_seed(0)
    cfg = WhisperConfig(d_model=64, encoder_layers=2, decoder_layers=2, encoder_attention_heads=4,
                        decoder_attention_heads=4, encoder_ffn_dim=128, decoder_ffn_dim=128, num_mel_bins=16,
                        max_source_positions=50, max_target_positions=20, vocab_size=100, pad_token_id=0,
                        bos_token_id=1, eos_token_id=2, decoder_start_token_id=1)
    m = WhisperModel(cfg).eval()
    with torch.no_grad():  # fp16-representable parameters, so BlazeLayerNorm's fp16 copies are exact
        for p in m.parameters():
            p.copy_(p.half().float())
    return m


def test_linear_groups():
    assert linear_group("WhisperEncoderLayer", "self_attn.q_proj") == "encoder_attn_qkv"
    assert linear_group("WhisperEncoderLayer", "self_attn.k_proj") == "encoder_attn_qkv"
    assert linear_group("WhisperEncoderLayer", "self_attn.out_proj") == "encoder_attn_out"
    assert linear_group("WhisperEncoderLayer", "fc2") == "encoder_ffn"
    assert linear_group("WhisperDecoderLayer", "self_attn.v_proj") == "decoder_self_attn"
    assert linear_group("WhisperDecoderLayer", "encoder_attn.out_proj") == "decoder_cross_attn"
    assert linear_group("WhisperDecoderLayer", "fc1") == "decoder_ffn"
    assert linear_group("WhisperEncoderLayer", "encoder_attn.q_proj") is None
    assert linear_group("SomethingElse", "fc1") is None


def test_patch_counts_and_fp16_outputs_unchanged():
    m = _tiny_model()
    feats = torch.randn(2, 16, 100, generator=torch.Generator().manual_seed(1))
    dec_ids = torch.tensor([[1, 5, 7], [1, 9, 3]])
    with torch.no_grad():
        ref = m(input_features=feats, decoder_input_ids=dec_ids).last_hidden_state
    counts = patch_layers(m, full_fp16())
    # 2 encoder layers x 6 linears + 2 decoder layers x 10 linears
    assert counts["patched_linears"] == 2 * 6 + 2 * 10
    # 2 encoder layers x 2 + encoder final, 2 decoder layers x 3 + decoder final
    assert counts["patched_layernorms"] == 2 * 2 + 1 + 2 * 3 + 1
    assert not any(k.startswith("fp8_") for k in counts)
    assert isinstance(m.encoder.layers[0].self_attn.q_proj, BlazeLinear)
    assert isinstance(m.decoder.layers[1].encoder_attn.out_proj, BlazeLinear)
    assert isinstance(m.encoder.layer_norm, BlazeLayerNorm)
    with torch.no_grad():
        out = m(input_features=feats, decoder_input_ids=dec_ids).last_hidden_state
    assert torch.equal(out, ref)


def test_patch_without_layernorms():
    m = _tiny_model()
    counts = patch_layers(m, full_fp16(), layernorms=False)
    assert counts["patched_layernorms"] == 0
    assert isinstance(m.encoder.layer_norm, torch.nn.LayerNorm)


def test_stacked_cross_kv_runs_one_projection_per_input():
    """k_proj / v_proj halves of a StackedKVProjection: one stacked linear per input tensor,
    the halves equal the separate projections, the cache is released once both were served
    and an in-place change of the input between the halves forces a new projection."""
    import torch.nn as nn
    from whisper_blaze_b200.modules import StackedKVProjection
    from whisper_blaze_b200.precision import LayerPrecision
    torch.manual_seed(0)
    lin_k, lin_v = nn.Linear(64, 48, bias=False), nn.Linear(64, 40)
    kv = StackedKVProjection(lin_k, lin_v, LayerPrecision())  # fp16 precision: the F.linear branch
    calls = []
    orig = kv.linear.forward
    kv.linear.forward = lambda x: (calls.append(x.shape), orig(x))[1]
    k_half, v_half = kv.half(0), kv.half(1)
    x = torch.randn(2, 10, 64)
    with torch.no_grad():
        k, v = k_half(x), v_half(x)
        assert len(calls) == 1 and kv._cache is None
        assert k.shape == (2, 10, 48) and v.shape == (2, 10, 40)
        torch.testing.assert_close(k, lin_k(x), rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(v, lin_v(x), rtol=1e-5, atol=1e-5)
        k.view(2, -1, 6, 8)  # HF views the half per head; a strided half must allow it
        x2 = x.clone()
        k_half(x2), v_half(x2)
        assert len(calls) == 2
        x3 = torch.randn(2, 10, 64)
        k_half(x3)
        x3.add_(1.0)  # modified in place between the two halves
        v3 = v_half(x3)
        assert len(calls) == 4  # the k half's projection, then a new one for the changed input
        torch.testing.assert_close(v3, lin_v(x3), rtol=1e-5, atol=1e-5)
