"""GPU parity of the FP8 encoder stack against the CPU oracle.

Both attention back ends of the stack (the tcgen05 kernel and torch SDPA) are covered.
Stage-wise, teacher-forced: every stage of a layer is recomputed by the oracle
from the GPU's own input to that stage and held to that stage's gate
(LayerNorm 1e-3 abs / fp16 ulp; fp8 bytes exact for the GPU's scale, scale
within 1 ulp of the IEEE quotient of the exact amax; each GEMM max relative
error <= 1e-2; attention <= 1e-2). End to end, FP8 rounding flips triggered
by last-bit differences upstream make per-element comparison after several
layers chaotic, so the whole stack is held to statistical gates instead
(cosine similarity and mean absolute error).
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from conftest import randn_f16
from oracle import encoder as ref_encoder
from oracle import fp8, gemm, norm
from whisper_blaze_b200.encoder import EncoderConfig, FP8EncoderStack, random_layer_weights

pytestmark = pytest.mark.gpu


def _layers(cfg, n, seed):
    g = torch.Generator().manual_seed(seed)
    return [random_layer_weights(cfg, g) for _ in range(n)]


def _check_ln(out, ref):
    err = (out.float().cpu() - ref).abs()
    assert (err <= norm.ln_tolerance(ref)).all(), f"LN max err {err.max().item():.3e}"


def _check_q(x16, q, s):
    """bytes exact for the GPU's scale; the scale within 1 ulp of IEEE amax/448 of the same tensor."""
    x = x16.cpu().numpy()
    s = np.float32(s.item())
    ieee = fp8.scale_from_amax(fp8.amax_f16(x), fp8.E4M3)
    assert abs(int(s.view(np.int32)) - int(ieee.view(np.int32))) <= 1, (s, ieee)
    assert np.array_equal(q.cpu().numpy(), fp8.quantise_with_scale(x, s, fp8.E4M3))


def _check_gemm(y, ref32):
    rel = gemm.rel_error(y, ref32)
    assert rel <= 1e-2, f"GEMM relative error {rel:.3e}"


@pytest.mark.parametrize("attention", ["wbk", "sdpa"])
@pytest.mark.parametrize("B,S", [(2, 64), (1, 1500)])
def test_layer_stagewise_parity(cuda_device, B, S, attention):
    cfg = EncoderConfig(layers=1, seq_len=S)
    stack = FP8EncoderStack(cfg, _layers(cfg, 1, 5), cuda_device, attention=attention)
    L = stack.layers[0]
    h = randn_f16((B, S, cfg.d_model), 6)
    cap = []
    stack.forward(h.to(cuda_device), capture=cap)
    c = {k: v.cpu() for k, v in cap[0].items() if torch.is_tensor(v)}
    f32 = lambda t: float(t.item())  # noqa: E731
    cpu = lambda t: t.cpu()  # noqa: E731

    _check_ln(c["ln1"], norm.layernorm_ref(c["in"], None, cpu(L.ln1_g), cpu(L.ln1_b)))
    _check_q(c["ln1"], c["ln1_q"], c["ln1_s"])
    _check_gemm(c["qkv"], gemm.gemm_fp8_ref_f32(c["ln1_q"], f32(c["ln1_s"]), cpu(L.w_qkv), f32(L.s_qkv),
                                                cpu(L.b_qkv)))
    H, Dh = cfg.heads, cfg.head_dim
    q, k, v = (c["qkv"].float().view(B, S, 3, H, Dh)[:, :, i].transpose(1, 2) for i in range(3))
    attn_ref = F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(B * S, cfg.d_model)
    assert gemm.rel_error(c["attn"], attn_ref) <= 1e-2
    _check_q(c["attn"], c["attn_q"], c["attn_s"])
    _check_gemm(c["h2"], gemm.gemm_fp8_ref_f32(c["attn_q"], f32(c["attn_s"]), cpu(L.w_o), f32(L.s_o), cpu(L.b_o),
                                               c["in"].view(B * S, -1), gemm.EPI_RESIDUAL))
    _check_ln(c["ln2"], norm.layernorm_ref(c["h2"], None, cpu(L.ln2_g), cpu(L.ln2_b)))
    _check_q(c["ln2"], c["ln2_q"], c["ln2_s"])
    _check_gemm(c["fc1"], gemm.gemm_fp8_ref_f32(c["ln2_q"], f32(c["ln2_s"]), cpu(L.w_fc1), f32(L.s_fc1),
                                                cpu(L.b_fc1)))
    # GELU runs inside the quantiser on the fp16 fc1 output; its amax comes from the GEMM's max key
    from test_gpu_quant import _check_gelu_quant
    _check_gelu_quant(c["fc1"], c["fc1_q"], c["fc1_s"])
    _check_gemm(c["out"], gemm.gemm_fp8_ref_f32(c["fc1_q"], f32(c["fc1_s"]), cpu(L.w_fc2), f32(L.s_fc2),
                                                cpu(L.b_fc2), c["h2"], gemm.EPI_RESIDUAL_CLAMP))


@pytest.mark.parametrize("attention", ["wbk", "sdpa"])
def test_two_layer_stack_statistics(cuda_device, attention):
    cfg = EncoderConfig(layers=2, seq_len=64)
    layers = _layers(cfg, 2, 5)
    stack = FP8EncoderStack(cfg, layers, cuda_device, attention=attention)
    h = randn_f16((2, 64, cfg.d_model), 6)
    y = stack.forward(h.to(cuda_device)).float().cpu().view(-1)
    ref = ref_encoder.encoder_stack_ref(h, [ref_encoder.quantise_layer(lw) for lw in layers], cfg.heads)
    ref = ref.float().view(-1)
    cos = F.cosine_similarity(y, ref, dim=0).item()
    mae = (y - ref).abs().mean().item() / ref.abs().mean().item()
    assert cos >= 0.999, f"cosine similarity {cos:.5f}"
    assert mae <= 0.03, f"relative mean abs error {mae:.4f}"


def test_stack_is_deterministic_and_host_path_agrees(cuda_device):
    cfg = EncoderConfig(layers=3, seq_len=128)
    stack = FP8EncoderStack(cfg, _layers(cfg, 3, 9), cuda_device)
    h = randn_f16((4, 128, cfg.d_model), 10)
    y1 = stack.forward(h.to(cuda_device)).clone()
    y2 = stack.forward(h.to(cuda_device)).clone()
    assert torch.equal(y1, y2)
    y3 = stack.forward_host(h.pin_memory())
    assert torch.equal(y3, y1.cpu())
    assert torch.isfinite(y1.float()).all()


def test_sliced_batch_matches_whole_batch(cuda_device):
    """Running the batch through the stack a few chunks at a time gives the same bits
    as one pass: per-tensor scales are per slice in both cases only if each slice is
    quantised on its own, so compare slice by slice against single-slice runs."""
    cfg = EncoderConfig(layers=2, seq_len=64)
    layers = _layers(cfg, 2, 11)
    sliced = FP8EncoderStack(cfg, layers, cuda_device, slice_chunks=2)
    whole = FP8EncoderStack(cfg, layers, cuda_device)
    h = randn_f16((5, 64, cfg.d_model), 12).to(cuda_device)
    y = sliced.forward(h).clone()
    for b0 in range(0, 5, 2):
        y_ref = whole.forward(h[b0:b0 + 2].contiguous())
        assert torch.equal(y[b0:b0 + 2], y_ref)


@pytest.mark.parametrize("attention", ["wbk", "sdpa"])
def test_graphed_forward_matches_eager(cuda_device, attention):
    cfg = EncoderConfig(layers=2, seq_len=96)
    stack = FP8EncoderStack(cfg, _layers(cfg, 2, 13), cuda_device, slice_chunks=2, attention=attention)
    h = randn_f16((3, 96, cfg.d_model), 14).to(cuda_device)
    y_eager = stack.forward(h).clone()
    y1 = stack.forward_graphed(h).clone()
    y2 = stack.forward_graphed(h).clone()  # replay
    assert torch.equal(y1, y_eager) and torch.equal(y2, y_eager)
    y_host = stack.forward_host(h.cpu().pin_memory(), graphed=True)
    assert torch.equal(y_host, y_eager.cpu())


def test_forward_host_stream_matches_forward(cuda_device):
    """The pipelined host API (copy-in / compute / copy-out overlapped through two buffer
    pairs) returns, batch by batch, exactly what forward() returns on the same input."""
    cfg = EncoderConfig(layers=2, seq_len=64)
    stack = FP8EncoderStack(cfg, _layers(cfg, 2, 21), cuda_device)
    batches = [randn_f16((3, 64, cfg.d_model), 30 + i).pin_memory() for i in range(5)]
    outs = [torch.empty(b.shape, dtype=torch.float16).pin_memory() for b in batches]
    stack.forward_host_stream(batches, outs)
    torch.cuda.synchronize()
    for b, o in zip(batches, outs):
        assert torch.equal(o, stack.forward(b.to(cuda_device)).cpu())
    # None entries skip the copy-out; a second call reuses the buffers and graphs
    stack.forward_host_stream(batches[:2], [None, outs[0]])
    torch.cuda.synchronize()
    assert torch.equal(outs[0], stack.forward(batches[1].to(cuda_device)).cpu())
