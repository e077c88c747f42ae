"""GPU parity of the tcgen05 FP8 GEMM (calls go through the C ABI).

Shapes cover the three tile widths the host picks (64 for M <= 128, 128 when
256-wide tiles would leave SMs idle, 256 otherwise).

Gate (north star): max relative error <= 1e-2, defined as
max|y - ref| / max|ref| over the output, against the fp32 matmul of the same
dequantised operands (oracle/gemm.py); elementwise also
|y - ref| <= 1e-2 * |ref| + 1e-2 * rms(ref). Plus: every output element is
written (NaN-poisoned output buffer), results are bitwise deterministic, the
fused output amax is exact.
"""
import numpy as np
import pytest
import torch

from conftest import randn_f16
from oracle import fp8, gemm
from whisper_blaze_b200 import _lib, ops

pytestmark = pytest.mark.gpu

REL_GATE = 1e-2


def _operands(M, N, K, seed, dev, a_fmt="e4m3", w_fmt="e4m3", bias=True):
    x = randn_f16((M, K), seed)
    w = randn_f16((N, K), seed + 1, std=0.02)
    aq, sa = ops.quantise(x.to(dev), a_fmt)
    wq, sw = ops.quantise(w.to(dev), w_fmt)
    b = randn_f16((N,), seed + 2, std=0.02).to(dev) if bias else None
    return aq, sa, wq, sw, b


def _ref(aq, sa, wq, sw, b, res=None, epi=gemm.EPI_NONE, a_fmt="e4m3", w_fmt="e4m3"):
    return gemm.gemm_fp8_ref_f32(aq.cpu(), float(sa.item()), wq.cpu(), float(sw.item()),
                                 None if b is None else b.cpu(), None if res is None else res.cpu(), epi,
                                 fp8.FMT_NAMES[a_fmt], fp8.FMT_NAMES[w_fmt])


def _check(y, ref32):
    y32 = y.float().cpu()
    ref16 = ref32.half().float()
    rel = gemm.rel_error(y32, ref32)
    assert rel <= REL_GATE, f"max relative error {rel:.3e}"
    rms = ref32.pow(2).mean().sqrt().item()
    bad = (y32 - ref32).abs() > (1e-2 * ref32.abs() + 1e-2 * rms)
    assert not bad.any(), f"{bad.sum().item()} elements outside the elementwise gate"
    assert not torch.isnan(y32).any()
    return rel, (y32 - ref16).abs().max().item()


SHAPES = [
    # (M, N, K): encoder / decoder shapes and odd edges
    (1500, 5120, 1280),   # config 1 (fc1)
    (64, 1280, 1280), (64, 3840, 1280), (64, 5120, 1280),  # config 3 decoder step
    (1, 256, 128), (63, 8, 16), (65, 24, 48), (129, 264, 272), (300, 1000, 1280),
    (256, 1280, 5120),    # fc2 K
    (130, 136, 4096 + 16),  # K not a multiple of the 128-byte stage
    (4096, 2560, 1280),   # enough tiles for the 256-wide tile path
    (4224 + 7, 2568, 384),  # 256-wide tiles with ragged M and N edges
]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_bias_matches_oracle(cuda_device, M, N, K):
    aq, sa, wq, sw, b = _operands(M, N, K, M + N + K, cuda_device)
    out = torch.full((M, N), float("nan"), dtype=torch.float16, device=cuda_device)  # poisoned
    y = ops.gemm_fp8(aq, sa, wq, sw, b, out=out)
    _check(y, _ref(aq, sa, wq, sw, b))


def test_gemm_vocab_projection(cuda_device):
    """Config 3 logits shape: N = 51866 is not a multiple of 8 (unaligned rows, masked edge tile)."""
    M, N, K = 64, 51866, 1280
    aq, sa, wq, sw, _ = _operands(M, N, K, 9, cuda_device, bias=False)
    y = ops.gemm_fp8(aq, sa, wq, sw, None)
    _check(y, _ref(aq, sa, wq, sw, None))


# The skinny kernel (A resident in shared memory, weight-only ring) serves M <= 64 with at most
# 12 K blocks (K <= 1536) in the one-call linear, and plain GEMMs with more tiles than SMs. Its
# edges, with every epilogue, plus the first K past it: the linear's codes, scale and output
# equal the standalone quantiser and gemm_fp8 on those codes, which meet the oracle gate.
@pytest.mark.parametrize("epi,name", [(gemm.EPI_NONE, "none"), (gemm.EPI_GELU, "gelu"),
                                      (gemm.EPI_RESIDUAL, "residual"), (gemm.EPI_RESIDUAL_CLAMP, "residual_clamp")])
@pytest.mark.parametrize("M,N,K", [(64, 51866, 1280),   # vocab: 811 tiles on 148 CTAs, ragged unaligned N
                                   (33, 4000, 1536),    # 12 K blocks: the largest resident A
                                   (64, 1000, 1424),    # K % 128 != 0: per-block 2-D loads, zero-filled tail
                                   (2, 72, 16),         # one partial K block
                                   (64, 520, 1552)])    # 13 K blocks: the general kernel
def test_gemm_skinny_edges(cuda_device, epi, name, M, N, K):
    x = randn_f16((M, K), 71 + K).to(cuda_device)
    wq, sw = ops.quantise(randn_f16((N, K), 72 + K, std=0.02).to(cuda_device))
    b = randn_f16((N,), 73, std=0.02).to(cuda_device)
    res = randn_f16((M, N), 74).to(cuda_device) if epi in (gemm.EPI_RESIDUAL, gemm.EPI_RESIDUAL_CLAMP) else None
    aq, sa = ops.quantise(x)
    out = torch.full((M, N), float("nan"), dtype=torch.float16, device=cuda_device)
    y = ops.gemm_fp8(aq, sa, wq, sw, b, res, name, out=out)
    _check(y, _ref(aq, sa, wq, sw, b, res, epi))
    assert torch.equal(y, ops.gemm_fp8(aq, sa, wq, sw, b, res, name))  # deterministic
    y_lin, q_lin, s_lin = ops.linear_fp8(x, wq, sw, b, res, name)
    assert torch.equal(q_lin, aq) and torch.equal(s_lin, sa)
    assert torch.equal(y_lin.view(torch.int16), y.view(torch.int16))


@pytest.mark.parametrize("epi,name", [(gemm.EPI_GELU, "gelu"), (gemm.EPI_RESIDUAL, "residual"),
                                      (gemm.EPI_RESIDUAL_CLAMP, "residual_clamp")])
@pytest.mark.parametrize("M,N,K", [(384, 5120, 1280), (200, 1280, 1280), (77, 40, 64), (4096, 2560, 640)])
def test_gemm_epilogues(cuda_device, epi, name, M, N, K):
    aq, sa, wq, sw, b = _operands(M, N, K, 31 + M, cuda_device)
    res = randn_f16((M, N), 33).to(cuda_device) if epi != gemm.EPI_GELU else None
    if epi == gemm.EPI_RESIDUAL_CLAMP:
        res[0, :4] = torch.tensor([65504.0, -65504.0, 64000.0, 1.0], dtype=torch.float16)
    y = ops.gemm_fp8(aq, sa, wq, sw, b, res, name)
    _check(y, _ref(aq, sa, wq, sw, b, res, epi))


@pytest.mark.parametrize("a_fmt,w_fmt", [("e5m2", "e4m3"), ("e4m3", "e5m2"), ("e5m2", "e5m2")])
def test_gemm_e5m2_operands(cuda_device, a_fmt, w_fmt):
    M, N, K = 256, 512, 640
    aq, sa, wq, sw, b = _operands(M, N, K, 50, cuda_device, a_fmt, w_fmt)
    y = ops.gemm_fp8(aq, sa, wq, sw, b, a_format=a_fmt, w_format=w_fmt)
    _check(y, _ref(aq, sa, wq, sw, b, a_fmt=a_fmt, w_fmt=w_fmt))


def test_gemm_host_float_scales(cuda_device):
    import whisper_blaze_kernels as K
    x = randn_f16((200, 1280), 60).to(cuda_device)
    w = randn_f16((768, 1280), 61, std=0.02).to(cuda_device)
    aq, sa = K.quantise_e4m3(x)
    wq, sw = K.quantise_e4m3(w)
    y = K.gemm_fp8_e4m3(aq, sa, wq, sw)
    ref = gemm.gemm_fp8_ref_f32(aq.cpu(), sa, wq.cpu(), sw)
    _check(y, ref)


def test_gemm_deterministic_and_amax(cuda_device):
    M, N, K = 1500, 5120, 1280
    aq, sa, wq, sw, b = _operands(M, N, K, 70, cuda_device)
    amax = ops.new_amax_ws(cuda_device)
    y1 = ops.gemm_fp8(aq, sa, wq, sw, b, epilogue="gelu", out_amax=amax)
    y2 = ops.gemm_fp8(aq, sa, wq, sw, b, epilogue="gelu")
    assert torch.equal(y1, y2)
    assert amax.item() == y1.float().abs().max().half().view(torch.int16).item()


def test_blaze_linear_fp8(cuda_device):
    from whisper_blaze_b200.modules import BlazeLinear
    from whisper_blaze_b200.precision import fp8_e4m3
    w = randn_f16((1280, 1280), 80, std=0.02).to(cuda_device)
    b = randn_f16((1280,), 81, std=0.02).to(cuda_device)
    lin = BlazeLinear(w, b, fp8_e4m3().encoder_attn_out)
    x = randn_f16((3, 50, 1280), 82).to(cuda_device)
    y = lin(x)
    assert y.shape == (3, 50, 1280)
    xq, sx = fp8.quantise(x.cpu().numpy(), fp8.E4M3)
    ref = gemm.gemm_fp8_ref_f32(torch.from_numpy(xq).view(-1, 1280), sx, lin._w_fp8.cpu(), lin._w_scale.item(),
                                b.cpu())
    _check(y.view(-1, 1280), ref)


def test_no_device_error_recorded(cuda_device):
    assert _lib.device_error() == 0


def test_gemm_max_key_epilogue(cuda_device):
    """'bias_maxkey': output as 'none', and out_amax receives the order key of the largest output."""
    from oracle.gemm import order_key_f16
    M, N, K = 300, 1000, 1280
    aq, sa, wq, sw, b = _operands(M, N, K, 90, cuda_device)
    key = ops.new_amax_ws(cuda_device)
    y = ops.gemm_fp8(aq, sa, wq, sw, b, epilogue="bias_maxkey", out_amax=key)
    y_none = ops.gemm_fp8(aq, sa, wq, sw, b)
    assert torch.equal(y, y_none)
    assert key.item() == order_key_f16(float(y.float().max()))
    with pytest.raises(RuntimeError, match="requires out_amax"):
        ops.gemm_fp8(aq, sa, wq, sw, b, epilogue="bias_maxkey")


# ---- split-K for short-M (decoder-step) shapes

@pytest.mark.parametrize("M,N,K", [(32, 1280, 5120), (16, 1280, 5120), (8, 24, 2048), (1, 256, 8192),
                                   (17, 640, 4096 + 16), (64, 1280, 1280)])
@pytest.mark.parametrize("epi", ["none", "residual", "bias_maxkey"])
def test_gemm_split_k(cuda_device, M, N, K, epi):
    """K split over more CTAs than the 64-wide column tiles (every shape here but the last one
    splits): same gate as the unsplit GEMM, bitwise deterministic across calls, and the
    workspace is left reusable (tickets back at 0)."""
    from whisper_blaze_b200 import _lib
    need = _lib.lib().wbk_gemm_fp8_ws_bytes(M, N, K)
    aq, sa, wq, sw, b = _operands(M, N, K, 7 * M + N + K, cuda_device)
    res = randn_f16((M, N), 3).to(cuda_device) if epi == "residual" else None
    key = ops.new_amax_ws(cuda_device) if epi == "bias_maxkey" else None
    ws = torch.zeros(max(need, 1), dtype=torch.uint8, device=cuda_device)
    y1 = ops.gemm_fp8(aq, sa, wq, sw, b, res, epi, out_amax=key, workspace=ws)
    y2 = ops.gemm_fp8(aq, sa, wq, sw, b, res, epi, out_amax=key, workspace=ws)
    assert torch.equal(y1, y2)
    ref_epi = gemm.EPI_RESIDUAL if epi == "residual" else gemm.EPI_NONE
    _check(y1, _ref(aq, sa, wq, sw, b, res, ref_epi))
    y_unsplit = ops.gemm_fp8(aq, sa, wq, sw, b, res, epi, out_amax=key, split_k=False)
    _check(y_unsplit, _ref(aq, sa, wq, sw, b, res, ref_epi))
    if epi == "bias_maxkey":
        from oracle.gemm import order_key_f16
        assert key.item() == order_key_f16(float(y1.float().max()))
    if need > 0:
        # the sync words and the ticket block (first 256 B + 16 KB of the workspace) must be all zero again
        assert int(ws[:256 + 16384].view(torch.int32).abs().sum().item()) == 0
    assert _lib.device_error() == 0


def test_gemm_split_k_workspace_errors(cuda_device):
    from whisper_blaze_b200 import _lib
    M, N, K = 16, 1280, 5120
    need = _lib.lib().wbk_gemm_fp8_ws_bytes(M, N, K)
    assert need > 0
    assert _lib.lib().wbk_gemm_fp8_ws_bytes(4096, 1280, 1280) == 0  # large M: no split, no in-kernel quantise
    # M <= 128 without a split: only the in-kernel quantise's sync words (wbk_linear_fp8_f16)
    assert _lib.lib().wbk_gemm_fp8_ws_bytes(16, 1280, 1280) == 256  # short K: no split
    assert _lib.lib().wbk_gemm_fp8_ws_bytes(64, 1280, 5120) == 256  # M = 64: no split
    aq, sa, wq, sw, b = _operands(M, N, K, 5, cuda_device)
    small = torch.zeros(need // 2, dtype=torch.uint8, device=cuda_device)
    with pytest.raises(RuntimeError, match="workspace"):
        ops.gemm_fp8(aq, sa, wq, sw, b, workspace=small)


def test_gemm_split_k_shared_workspace_across_shapes(cuda_device):
    """One workspace serving several short-M shapes in turn (the decoder step does this):
    the partials of one shape must never land on another shape's tickets."""
    shapes = [(16, 3840, 2048), (32, 1280, 5120), (16, 2560, 5120), (64, 1280, 1280)]
    ops_ = []
    for i, (M, N, K) in enumerate(shapes):
        aq, sa, wq, sw, b = _operands(M, N, K, 100 + i, cuda_device)
        ops_.append((aq, sa, wq, sw, b, ops.gemm_fp8(aq, sa, wq, sw, b, split_k=False)))
    for _ in range(3):
        for aq, sa, wq, sw, b, ref in ops_:
            y = ops.gemm_fp8(aq, sa, wq, sw, b)
            assert gemm.rel_error(y.float().cpu(), ref.float().cpu()) <= 1e-2


_GENERAL_KERNEL_SCRIPT = r"""
import sys, torch
sys.path.insert(0, {tests!r})
from conftest import randn_f16
from whisper_blaze_b200 import ops
dev = torch.device("cuda:0")
outs = []
for (M, N, K, epi) in {cases!r}:
    x = randn_f16((M, K), M + K).to(dev)
    w = randn_f16((N, K), N, std=0.02).to(dev)
    b = randn_f16((N,), 5, std=0.02).to(dev)
    res = randn_f16((M, N), 6).to(dev) if epi.startswith("residual") else None
    wq, sw = ops.quantise(w)
    y, q, s = ops.linear_fp8(x, wq, sw, b, res, epi)
    y2 = ops.gemm_fp8(q, s, wq, sw, b, res, epi)
    outs.append((y.cpu(), q.cpu(), s.cpu(), y2.cpu()))
torch.save(outs, {path!r})
"""


def test_skinny_kernel_matches_general_kernel(cuda_device, tmp_path):
    """The skinny kernel (and its in-kernel quantise) gives bit-identical codes, scales and
    outputs to the general 64-wide kernel (WBK_GEMM_SKINNY=0, run in a subprocess)."""
    import os
    import subprocess
    import sys
    cases = [(64, 1280, 1280, "none"), (64, 3840, 1280, "residual"), (17, 640, 1296, "gelu"), (5, 51866, 1280, "none")]
    path = str(tmp_path / "general.pt")
    script = _GENERAL_KERNEL_SCRIPT.format(tests=os.path.dirname(os.path.abspath(__file__)), cases=cases, path=path)
    env = dict(os.environ, WBK_GEMM_SKINNY="0")
    subprocess.run([sys.executable, "-c", script], env=env, check=True, timeout=600)
    general = torch.load(path)
    for (M, N, K, epi), (yg, qg, sg, y2g) in zip(cases, general):
        x = randn_f16((M, K), M + K).to(cuda_device)
        w = randn_f16((N, K), N, std=0.02).to(cuda_device)
        b = randn_f16((N,), 5, std=0.02).to(cuda_device)
        res = randn_f16((M, N), 6).to(cuda_device) if epi.startswith("residual") else None
        wq, sw = ops.quantise(w)
        y, q, s = ops.linear_fp8(x, wq, sw, b, res, epi)
        y2 = ops.gemm_fp8(q, s, wq, sw, b, res, epi)
        assert torch.equal(q.cpu(), qg) and torch.equal(s.cpu(), sg), (M, N, K)
        assert torch.equal(y.cpu().view(torch.int16), yg.view(torch.int16)), (M, N, K, "linear")
        assert torch.equal(y2.cpu().view(torch.int16), y2g.view(torch.int16)), (M, N, K, "gemm")


# CTA-pair (256 x 256) residual epilogues load each 32 x 32 residual box by TMA into the store
# staging buffer and write the output over it. Ragged M leaves boxes partly and wholly past row M
# (zero fill, clipped store; at M = 4100 the second CTA of the last pair has no rows at all);
# N % 32 == 8 leaves a partial last chunk; N % 8 != 0 takes the per-thread loads and direct stores.
PAIR_RESIDUAL_SHAPES = [(4231, 2568, 384), (4100, 2560, 640), (4096, 2570, 384), (6000, 1280, 1280)]


@pytest.mark.parametrize("epi,name", [(gemm.EPI_RESIDUAL, "residual"), (gemm.EPI_RESIDUAL_CLAMP, "residual_clamp")])
@pytest.mark.parametrize("M,N,K", PAIR_RESIDUAL_SHAPES)
def test_gemm_pair_residual_edges(cuda_device, epi, name, M, N, K):
    aq, sa, wq, sw, b = _operands(M, N, K, 41 + N, cuda_device)
    res = randn_f16((M, N), 43).to(cuda_device)
    if epi == gemm.EPI_RESIDUAL_CLAMP:
        res[-1, -4:] = torch.tensor([65504.0, -65504.0, 64000.0, 1.0], dtype=torch.float16)
    out = torch.full((M + 1, N), float("nan"), dtype=torch.float16, device=cuda_device)  # one guard row
    y = ops.gemm_fp8(aq, sa, wq, sw, b, res, name, out=out[:M])
    _check(y, _ref(aq, sa, wq, sw, b, res, epi))
    assert torch.isnan(out[M]).all()  # nothing stored past row M


def test_pair_residual_tma_matches_thread_loads(cuda_device, tmp_path):
    """The TMA-loaded residual gives bit-identical outputs to the per-thread residual
    loads (WBK_GEMM_RES_TMA=0, run in a subprocess), ragged edges included."""
    import os
    import subprocess
    import sys
    cases = [(M, N, K, epi) for (M, N, K) in PAIR_RESIDUAL_SHAPES for epi in ("residual", "residual_clamp")]
    path = str(tmp_path / "thread_loads.pt")
    script = _GENERAL_KERNEL_SCRIPT.format(tests=os.path.dirname(os.path.abspath(__file__)), cases=cases, path=path)
    env = dict(os.environ, WBK_GEMM_RES_TMA="0")
    subprocess.run([sys.executable, "-c", script], env=env, check=True, timeout=600)
    other = torch.load(path)
    for (M, N, K, epi), (yg, qg, sg, y2g) in zip(cases, other):
        x = randn_f16((M, K), M + K).to(cuda_device)
        w = randn_f16((N, K), N, std=0.02).to(cuda_device)
        b = randn_f16((N,), 5, std=0.02).to(cuda_device)
        res = randn_f16((M, N), 6).to(cuda_device)
        wq, sw = ops.quantise(w)
        y, q, s = ops.linear_fp8(x, wq, sw, b, res, epi)
        y2 = ops.gemm_fp8(q, s, wq, sw, b, res, epi)
        assert torch.equal(q.cpu(), qg) and torch.equal(s.cpu(), sg), (M, N, K)
        assert torch.equal(y.cpu().view(torch.int16), yg.view(torch.int16)), (M, N, K, epi, "linear")
        assert torch.equal(y2.cpu().view(torch.int16), y2g.view(torch.int16)), (M, N, K, epi, "gemm")


# CTA pairs split the tiles of a partial last round into 2 or 4 narrower items (MMA N = 128 or
# 64; 74 pairs on a B200). Run with WBK_GEMM_BN=256 so every shape takes the pair kernel:
NARROW_CASES = [(11900, 1280, 1280, "residual"),      # 235 tiles = 3 rounds + 13 -> 52 quarter items; ragged M
                (6300, 1288, 640, "residual_clamp"),  # 150 tiles = 2 rounds + 2 -> quarters; N 8 past a tile
                (4100, 2560, 640, "none"),            # 170 tiles = 2 rounds + 22 -> 44 half items
                (2000, 1000, 1280, "gelu"),           # 32 tiles, no whole round -> 64 halves; N % 32 = 8
                (3000, 520, 256, "residual")]         # 36 tiles -> 72 halves


def test_gemm_pair_narrow_last_round(cuda_device, tmp_path):
    """Narrow last-round items meet the oracle gate and give bit-identical outputs to whole
    tiles (WBK_GEMM_NARROW=0): the same K-ordered MMA accumulation per output element."""
    import os
    import subprocess
    import sys
    tests = os.path.dirname(os.path.abspath(__file__))
    outs = {}
    for tag, extra in (("narrow", {}), ("whole", {"WBK_GEMM_NARROW": "0"})):
        path = str(tmp_path / f"{tag}.pt")
        script = _GENERAL_KERNEL_SCRIPT.format(tests=tests, cases=NARROW_CASES, path=path)
        env = dict(os.environ, WBK_GEMM_BN="256", **extra)
        subprocess.run([sys.executable, "-c", script], env=env, check=True, timeout=600)
        outs[tag] = torch.load(path)
    epi_code = {"none": gemm.EPI_NONE, "gelu": gemm.EPI_GELU, "residual": gemm.EPI_RESIDUAL,
                "residual_clamp": gemm.EPI_RESIDUAL_CLAMP}
    for (M, N, K, epi), (y, q, s, y2), (yw, qw, sw_, y2w) in zip(NARROW_CASES, outs["narrow"], outs["whole"]):
        w = randn_f16((N, K), N, std=0.02).to(cuda_device)
        b = randn_f16((N,), 5, std=0.02)
        res = randn_f16((M, N), 6) if epi.startswith("residual") else None
        wq, sw = ops.quantise(w)
        _check(y2, gemm.gemm_fp8_ref_f32(q, float(s.item()), wq.cpu(), float(sw.item()), b, res, epi_code[epi]))
        assert torch.equal(q, qw) and torch.equal(s, sw_)
        assert torch.equal(y2.view(torch.int16), y2w.view(torch.int16)), (M, N, K, epi)
        assert torch.equal(y.view(torch.int16), y2.view(torch.int16))


@pytest.mark.parametrize("M,N,K", [(1500, 5120, 1280), (64, 1280, 1280), (300, 1000, 1296)])
def test_gemm_vs_reference_gpu_linear_path(cuda_device, M, N, K):
    """Against the reference's own GPU path for an FP8 linear (BlazeLinear.forward,
    whisper_blaze/model.py:80-109): quantise x, dequantise both operands to fp16
    (dequantise_e4m3, bit-identical to the reference kernel), then F.linear (cuBLAS fp16).
    The operands differ only by the fp16 rounding of the dequantised values, so the
    north-star gate (max relative error <= 1e-2) applies; the error is printed."""
    import whisper_blaze_kernels as K_
    x = randn_f16((M, K), 91 + M).to(cuda_device)
    w = randn_f16((N, K), 92 + N, std=0.02).to(cuda_device)
    b = randn_f16((N,), 93, std=0.02).to(cuda_device)
    aq, sa = K_.quantise_e4m3(x)
    wq, sw = K_.quantise_e4m3(w)
    a16 = K_.dequantise_e4m3(aq, sa, [M, K])
    w16 = K_.dequantise_e4m3(wq, sw, [N, K])
    y_ref_path = torch.nn.functional.linear(a16, w16, b).float()
    y = ops.gemm_fp8(aq, sa, wq, sw, b).float()
    rel = ((y - y_ref_path).abs().max() / y_ref_path.abs().max()).item()
    print(f"\nFP8 GEMM vs reference GPU path (fp16 dequantise + cuBLAS) {M}x{N}x{K}: max relative error {rel:.3e}")
    assert rel <= REL_GATE
