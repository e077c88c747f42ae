"""GPU parity at the sizes the benchmark numbers come from.

The other GPU tests pin the kernels on shapes the CPU oracle checks in full.
These run the shapes of BASELINE configs 2 and 4, the FFN GEMMs of the
config-5 stack at one GPU (M = 96 000 tokens) and at eight (M = 12 000 per
rank), and stage-wise teacher-forced layers of the benchmark's own weights at
the benchmark's batch (64 chunks x 1500 frames, and the 8-chunk shard of one
rank at 8 GPUs), so the persistent schedule's many rounds, the tile-index and
TMA-coordinate arithmetic at these sizes and the ragged last tiles are covered.

The gates are the ones every parity test here uses (oracle/gemm.py, oracle/fp8.py,
oracle/norm.py): GEMM max relative error <= 1e-2 plus the elementwise gate,
LayerNorm 1e-3 abs (one fp16 ulp where the fp16 grid is coarser), fp8 bytes
bit-exact for the kernel's scale with the scale within 1 ulp of the IEEE
quotient of the exact amax. To keep the CPU oracle's matmuls to seconds, each
GEMM is compared on a seeded sample of 4096 output rows that always includes
the first and last 256 rows (the last, partial tiles); amax and scales are
always taken over the whole tensor.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import fp8, gemm, norm
from whisper_blaze_b200 import ops
from whisper_blaze_b200.encoder import (EncoderConfig, FP8EncoderStack, synthetic_hidden,
                                        synthetic_stack_weights)

pytestmark = pytest.mark.gpu

SAMPLE_ROWS = 4096


def _rows(M, seed, n=SAMPLE_ROWS):
    """Sorted row indices: the first and last 256 rows and a seeded random rest."""
    edge = np.r_[np.arange(min(256, M)), np.arange(max(0, M - 256), M)]
    rng = np.random.default_rng(seed)
    rest = rng.choice(M, size=min(M, n), replace=False)
    return torch.from_numpy(np.unique(np.r_[edge, rest])[:n + 512].astype(np.int64))


def _randn(shape, seed, dev, std=1.0):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    return (torch.randn(*shape, generator=g, device=dev, dtype=torch.float32) * std).half()


def _check_gemm(y, ref32):
    """max relative error <= 1e-2 and |y - ref| <= 1e-2 |ref| + 1e-2 rms(ref), elementwise."""
    y32 = y.float().cpu()
    rel = gemm.rel_error(y32, ref32)
    assert rel <= 1e-2, f"max relative error {rel:.3e}"
    rms = ref32.pow(2).mean().sqrt().item()
    bad = (y32 - ref32).abs() > (1e-2 * ref32.abs() + 1e-2 * rms)
    assert not bad.any(), f"{bad.sum().item()} elements outside the elementwise gate"
    assert torch.isfinite(y32).all()
    return rel


def _gemm_rows(y, rows, aq, sa, wq, sw, b, res=None, epi=gemm.EPI_NONE):
    ref = gemm.gemm_fp8_ref_f32(aq[rows.to(aq.device)].cpu(), float(sa.item()), wq.cpu(), float(sw.item()),
                                None if b is None else b.cpu(),
                                None if res is None else res[rows.to(res.device)].cpu(), epi)
    return _check_gemm(y[rows.to(y.device)], ref)


def _check_quant(x16, q, s, rows):
    """Scale within 1 ulp of the IEEE quotient of the whole tensor's exact amax; bytes
    bit-exact for the kernel's scale on the sampled rows."""
    x = x16.cpu().numpy()
    s = np.float32(s.item())
    ieee = fp8.scale_from_amax(fp8.amax_f16(x), fp8.E4M3)
    assert abs(int(s.view(np.int32)) - int(ieee.view(np.int32))) <= 1, (s, ieee)
    r = rows.numpy()
    assert np.array_equal(q.cpu().numpy()[r], fp8.quantise_with_scale(x[r], s, fp8.E4M3))


def _check_gelu_quant(y16, q, s, rows):
    """codes of fp16(gelu(y)): scale from the whole tensor's GELU amax (one fp16 ulp of the
    amax: the GPU's erf is A&S 7.1.26, the oracle's exact), codes on the sampled rows
    equal for all but a few elements, and those one fp8 step apart at most."""
    g_all = gemm.gelu_f16(y16.cpu())
    s_gpu = np.float32(s.item())
    s_ref = fp8.scale_from_amax(fp8.amax_f16(g_all.numpy()), fp8.E4M3)
    assert abs(s_gpu / s_ref - 1.0) <= 2.0 ** -10, (s_gpu, s_ref)
    r = rows.numpy()
    q_ref = fp8.quantise_with_scale(g_all.numpy()[r], s_gpu, fp8.E4M3)
    qs = q.cpu().numpy()[r]
    diff = qs != q_ref
    assert diff.mean() <= 5e-3, f"{diff.mean():.4%} of fp8 codes differ"
    a = fp8.decode(qs[diff], fp8.E4M3).astype(np.float64)
    b = fp8.decode(q_ref[diff], fp8.E4M3).astype(np.float64)
    assert (np.abs(a - b) <= np.maximum(np.abs(a), np.abs(b)) * 2.0 ** -3 + 2.0 ** -9).all()


# --------------------------------------------------------------- config 2

def test_config2_layer_gemm_set_m24000(cuda_device):
    """The encoder layer's four GEMMs at batch 16 (M = 24 000), as the stack runs them:
    qkv (bias), out_proj (bias + residual), fc1 (bias + max key) -> GELU-quantise,
    fc2 (bias + residual + fp16 clamp)."""
    dev = cuda_device
    M, D, Fd = 24000, 1280, 5120
    rows = _rows(M, 1)
    x = _randn((M, D), 10, dev)
    h = _randn((M, D), 11, dev)
    xq, sx = ops.quantise(x)
    shapes = (("qkv", (3 * D, D)), ("o", (D, D)), ("fc1", (Fd, D)), ("fc2", (D, Fd)))
    w = {n: ops.quantise(_randn(shape, 20 + i, dev, 0.02)) for i, (n, shape) in enumerate(shapes)}
    b = {n: _randn((shape[0],), 30 + i, dev, 0.02) for i, (n, shape) in enumerate(shapes)}
    qkv = ops.gemm_fp8(xq, sx, *w["qkv"], b["qkv"])
    _gemm_rows(qkv, rows, xq, sx, *w["qkv"], b["qkv"])
    h2 = ops.gemm_fp8(xq, sx, *w["o"], b["o"], residual=h, epilogue="residual")
    _gemm_rows(h2, rows, xq, sx, *w["o"], b["o"], h, gemm.EPI_RESIDUAL)
    key = torch.zeros(1, dtype=torch.int32, device=dev)
    f = ops.gemm_fp8(xq, sx, *w["fc1"], b["fc1"], epilogue="bias_maxkey", out_amax=key)
    _gemm_rows(f, rows, xq, sx, *w["fc1"], b["fc1"])
    assert int(key.item()) == gemm.order_key_f16(float(f.float().max().item())), "fc1 max key"
    fq, sf = ops.quantise_gelu(f, key)
    _check_gelu_quant(f, fq, sf, rows)
    out = ops.gemm_fp8(fq, sf, *w["fc2"], b["fc2"], residual=h2, epilogue="residual_clamp")
    _gemm_rows(out, rows, fq, sf, *w["fc2"], b["fc2"], h2, gemm.EPI_RESIDUAL_CLAMP)


# --------------------------------------------------------------- config 4

def _ref_module():
    from oracle import build_ref
    try:
        return build_ref.load()
    except ImportError:
        return None


def test_config4_crossattn_kv_and_quantise_m48000(cuda_device):
    """Stacked cross-attention K/V over 32 x 1500 encoder frames: the standalone quantise of the
    48 000 x 1280 activation (bit-exact scale and bytes against the reference's own CUDA
    quantiser when its build is present, and against the oracle's rule), then the
    48 000 x 2560 x 1280 GEMM."""
    dev = cuda_device
    M, K, N = 48000, 1280, 2560
    rows = _rows(M, 2)
    x = _randn((M, K), 40, dev)
    xq, sx = ops.quantise(x)
    _check_quant(x, xq, sx, rows)
    R = _ref_module()
    if R is not None:
        q_ref, s_ref = R.quantise_e4m3(x)
        assert np.float32(sx.item()).view(np.int32) == np.float32(s_ref).view(np.int32)
        assert torch.equal(xq, q_ref.view(torch.uint8).to(dev)), "bytes differ from the reference kernel"
    wq, sw = ops.quantise(_randn((N, K), 41, dev, 0.02))
    b = _randn((N,), 42, dev, 0.02)
    y = ops.gemm_fp8(xq, sx, wq, sw, b)
    _gemm_rows(y, rows, xq, sx, wq, sw, b)


# ------------------------------------------------ FFN GEMMs of the stack

@pytest.mark.parametrize("M", [96000, 12000])
def test_stack_ffn_gemms(cuda_device, M):
    """fc1 (1280 -> 5120, bias + max key) and fc2 (5120 -> 1280, bias + residual + clamp) at
    the stack's token counts on one GPU (64 chunks) and on each of eight (8 chunks)."""
    dev = cuda_device
    D, Fd = 1280, 5120
    rows = _rows(M, 3 + M)
    aq, sa = ops.quantise(_randn((M, D), 50, dev))
    w1, s1 = ops.quantise(_randn((Fd, D), 51, dev, 0.02))
    b1 = _randn((Fd,), 52, dev, 0.02)
    key = torch.zeros(1, dtype=torch.int32, device=dev)
    f = ops.gemm_fp8(aq, sa, w1, s1, b1, epilogue="bias_maxkey", out_amax=key)
    _gemm_rows(f, rows, aq, sa, w1, s1, b1)
    assert int(key.item()) == gemm.order_key_f16(float(f.float().max().item()))
    del f
    fq, sf = ops.quantise(_randn((M, Fd), 53, dev))
    w2, s2 = ops.quantise(_randn((D, Fd), 54, dev, 0.02))
    b2 = _randn((D,), 55, dev, 0.02)
    res = _randn((M, D), 56, dev)
    out = ops.gemm_fp8(fq, sf, w2, s2, b2, residual=res, epilogue="residual_clamp")
    _gemm_rows(out, rows, fq, sf, w2, s2, b2, res, gemm.EPI_RESIDUAL_CLAMP)


# ----------------------------------- stage-wise layers of the benchmark

@pytest.fixture(scope="module")
def bench_stack(cuda_device):
    cfg = EncoderConfig()
    return cfg, FP8EncoderStack(cfg, synthetic_stack_weights(cfg, cuda_device), cuda_device)


@pytest.mark.parametrize("chunks,layer", [(64, 0), (64, 31), (8, 0)])
def test_bench_layer_stagewise(cuda_device, bench_stack, chunks, layer):
    """Layer `layer` of the benchmark's 32-layer stack (its weights, its input: 64 chunks on one
    GPU, or rank 0's 8-chunk shard at eight), every stage recomputed by the oracle from the
    GPU's own input to that stage."""
    cfg, stack = bench_stack
    B, S, D = chunks, cfg.seq_len, cfg.d_model
    T = B * S
    x = synthetic_hidden(B, cfg, cuda_device, seed=99)
    cap = []
    stack.forward(x, capture=cap, capture_layers={layer})
    assert len(cap) == 1 and cap[0]["layer"] == layer
    c = cap[0]
    L = stack.layers[layer]
    rows = _rows(T, 7 + layer)
    rd = rows.to(cuda_device)
    cpu = lambda t: t.cpu()  # noqa: E731

    ln1 = norm.layernorm_ref(c["in"].view(T, D)[rd].cpu(), None, cpu(L.ln1_g), cpu(L.ln1_b))
    err = (c["ln1"].view(T, D)[rd].float().cpu() - ln1).abs()
    assert (err <= norm.ln_tolerance(ln1)).all(), f"LN1 max err {err.max().item():.3e}"
    _check_quant(c["ln1"].view(T, D), c["ln1_q"], c["ln1_s"], rows)
    _gemm_rows(c["qkv"], rows, c["ln1_q"], c["ln1_s"], L.w_qkv, L.s_qkv, L.b_qkv)

    # attention of the first and last chunk, fp32 SDPA on the GPU's fp16 q/k/v
    H, Dh = cfg.heads, cfg.head_dim
    for b in sorted({0, B - 1}):
        qkv_b = c["qkv"].view(B, S, 3, H, Dh)[b].float().cpu()
        q, k, v = (qkv_b[:, i].transpose(0, 1) for i in range(3))
        a_ref = F.scaled_dot_product_attention(q, k, v).transpose(0, 1).reshape(S, D)
        rel = gemm.rel_error(c["attn"].view(B, S, D)[b], a_ref)
        assert rel <= 1e-2, f"attention chunk {b}: relative error {rel:.3e}"
    _check_quant(c["attn"].view(T, D), c["attn_q"], c["attn_s"], rows)
    _gemm_rows(c["h2"], rows, c["attn_q"], c["attn_s"], L.w_o, L.s_o, L.b_o, c["in"].view(T, D), gemm.EPI_RESIDUAL)

    ln2 = norm.layernorm_ref(c["h2"][rd].cpu(), None, cpu(L.ln2_g), cpu(L.ln2_b))
    err = (c["ln2"][rd].float().cpu() - ln2).abs()
    assert (err <= norm.ln_tolerance(ln2)).all(), f"LN2 max err {err.max().item():.3e}"
    _check_quant(c["ln2"], c["ln2_q"], c["ln2_s"], rows)
    _gemm_rows(c["fc1"], rows, c["ln2_q"], c["ln2_s"], L.w_fc1, L.s_fc1, L.b_fc1)
    _check_gelu_quant(c["fc1"], c["fc1_q"], c["fc1_s"], rows)
    _gemm_rows(c["out"], rows, c["fc1_q"], c["fc1_s"], L.w_fc2, L.s_fc2, L.b_fc2, c["h2"],
               gemm.EPI_RESIDUAL_CLAMP)
