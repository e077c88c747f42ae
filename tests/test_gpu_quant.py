"""GPU parity of the quantiser / dequantiser (calls go through the C ABI).

Gate: FP8 bytes and scales bit-exact.
  * bytes: against the oracle's element rule (oracle/fp8.py), given the scale;
  * scale: against the reference CUDA quantiser's own scale — live from
    oracle/_ref when that build is present, and always against the golden table
    of the reference scale for every positive finite fp16 amax
    (tests/golden/ref_scale_table.npz) — and within 1 ulp of the IEEE quotient.
"""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN_DIR, randn_f16
from oracle import fp8
from whisper_blaze_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def _special_values(n=4096, seed=7):
    g = torch.Generator().manual_seed(seed)
    bits = torch.randint(0, 65536, (n,), generator=g, dtype=torch.int32).to(torch.int16)
    x = bits.view(torch.float16).clone()
    x[:8] = torch.tensor([0.0, -0.0, float("nan"), float("inf"), -float("inf"), 65504.0, -65504.0, 6e-8])
    return x


def _cases():
    yield "randn_1500x1280", randn_f16((1500, 1280), 100)
    yield "weights_5120x1280", randn_f16((5120, 1280), 101, std=0.02)
    yield "randn_64x1280", randn_f16((64, 1280), 102)
    yield "ragged_7", randn_f16((7,), 103)
    yield "ragged_13", randn_f16((13,), 104)
    yield "ragged_4099", randn_f16((4099,), 105)
    yield "single", torch.tensor([0.75], dtype=torch.float16)
    yield "zeros", torch.zeros(4096, dtype=torch.float16)
    yield "specials", _special_values()
    yield "finite_no_inf", torch.nan_to_num(_special_values(seed=8), posinf=0.0, neginf=0.0)
    yield "tiny", (randn_f16((1024,), 106) * 1e-6).half()
    yield "huge", (randn_f16((1024,), 107) * 20000).half()


CASES = list(_cases())


@pytest.mark.parametrize("fmt_name", ["e4m3", "e5m2"])
@pytest.mark.parametrize("name,x", CASES, ids=[c[0] for c in CASES])
def test_quantise_bit_exact(cuda_device, name, x, fmt_name):
    fmt = fp8.FMT_NAMES[fmt_name]
    q, s = ops.quantise(x.to(cuda_device), fmt_name)
    q, s = q.cpu().numpy(), np.float32(s.item())
    # the scale: IEEE quotient within 1 ulp (exact equality with the reference is checked below)
    ieee = fp8.scale_from_amax(fp8.amax_f16(x.numpy()), fmt)
    if np.isfinite(ieee):
        assert abs(int(s.view(np.int32)) - int(ieee.view(np.int32))) <= 1, (s, ieee)
    else:
        assert s == ieee
    # the bytes: exactly the oracle's element rule for that scale
    q_ref = fp8.quantise_with_scale(x.numpy(), s, fmt)
    assert np.array_equal(q, q_ref), f"{np.count_nonzero(q != q_ref)} bytes differ"


@pytest.mark.parametrize("fmt_name", ["e4m3", "e5m2"])
def test_dequantise_bit_exact(cuda_device, fmt_name):
    fmt = fp8.FMT_NAMES[fmt_name]
    codes = torch.arange(256, dtype=torch.uint8).repeat(41)[:10001]  # ragged, every code
    for scale in (1.0, 0.0123, 146.2, 3.3e-9):
        out = ops.dequantise(codes.to(cuda_device), scale, [codes.numel()], fmt_name).cpu().numpy()
        ref = fp8.dequantise(codes.numpy(), scale, fmt)
        # NaN payloads may differ between the GPU and numpy; NaN positions and every other bit must not
        nan = np.isnan(ref)
        assert np.array_equal(np.isnan(out), nan)
        assert np.array_equal(out[~nan].view(np.uint16), ref[~nan].view(np.uint16))


def test_scale_stays_on_device_and_matches_host_api(cuda_device):
    import whisper_blaze_kernels as K
    x = randn_f16((512, 512), 110).to(cuda_device)
    q_host, s_host = K.quantise_e4m3(x)
    q_dev, s_dev = K.quantise_e4m3_dev(x)
    assert isinstance(s_host, float) and s_dev.is_cuda and s_dev.dtype == torch.float32
    assert torch.equal(q_host, q_dev) and np.float32(s_host) == np.float32(s_dev.item())


# ---- the reference's own quantiser tests (tests/test_kernels.py:42-79) on the B200 kernels

def test_ref_suite_roundtrips(cuda_device):
    import whisper_blaze_kernels as K
    x = torch.randn(128, 512, dtype=torch.float16, device=cuda_device)
    fp, scale = K.quantise_e4m3(x)
    assert fp.shape == x.shape and scale > 0
    x = torch.randn(512, 512, dtype=torch.float16, device=cuda_device)
    fp, scale = K.quantise_e4m3(x)
    xh = K.dequantise_e4m3(fp, scale, list(x.shape))
    assert torch.allclose(x.float(), xh.float(), atol=0.1, rtol=0.2)
    fp, scale = K.quantise_e5m2(x)
    xh = K.dequantise_e5m2(fp, scale, list(x.shape))
    assert torch.allclose(x.float(), xh.float(), atol=0.2, rtol=0.3)
    z = torch.zeros(64, 64, dtype=torch.float16, device=cuda_device)
    fp, scale = K.quantise_e4m3(z)
    assert torch.allclose(K.dequantise_e4m3(fp, scale, [64, 64]).float(), z.float(), atol=1e-6)


def test_dequantise_shape_mismatch_raises(cuda_device):
    import whisper_blaze_kernels as K
    fp, s = K.quantise_e4m3(torch.randn(8, 8, dtype=torch.float16, device=cuda_device))
    with pytest.raises(RuntimeError, match="holds"):
        K.dequantise_e4m3(fp, s, [8, 9])


# ---- against the reference scale, every positive finite fp16 amax

def _our_scale_table(cuda_device, amax_bits: np.ndarray, fmt: int) -> np.ndarray:
    L = _lib.lib()
    n = len(amax_bits)
    amax = torch.from_numpy(amax_bits.astype(np.int32)).to(cuda_device)
    scales = torch.zeros(n, dtype=torch.float32, device=cuda_device)
    dummy = torch.zeros(8, dtype=torch.float16, device=cuda_device)
    dq = torch.zeros(8, dtype=torch.uint8, device=cuda_device)
    stream = _lib.stream_of(dummy)
    a0, s0 = amax.data_ptr(), scales.data_ptr()
    for i in range(n):  # n == 0: only the scale is produced
        _lib.check(L.wbk_quantise_from_amax_f16(dummy.data_ptr(), 0, fmt, a0 + 4 * i, dq.data_ptr(), s0 + 4 * i,
                                                stream), "scale table")
    return scales.cpu().numpy()


def test_scale_table_matches_reference_golden(cuda_device):
    path = os.path.join(GOLDEN_DIR, "ref_scale_table.npz")
    if not os.path.exists(path):
        pytest.fail(f"{path} missing (generate with tests/golden/make_golden.py)")
    g = np.load(path)
    bits = g["amax_bits"].astype(np.uint16)
    for fmt_name, fmt in fp8.FMT_NAMES.items():
        ours = _our_scale_table(cuda_device, bits, fmt)
        ref = g[f"scale_{fmt_name}"].astype(np.float32)
        bad = np.flatnonzero(ours.view(np.int32) != ref.view(np.int32))
        assert bad.size == 0, f"{fmt_name}: {bad.size} scales differ from the reference, e.g. amax bits {bits[bad[:5]]}"


def test_quantise_matches_reference_golden_bytes(cuda_device):
    path = os.path.join(GOLDEN_DIR, "ref_quantise.npz")
    if not os.path.exists(path):
        pytest.fail(f"{path} missing (generate with tests/golden/make_golden.py)")
    g = np.load(path)
    for name in sorted({k.split("__")[0] for k in g.files}):
        x = torch.from_numpy(g[f"{name}__x"])
        for fmt_name in ("e4m3", "e5m2"):
            q, s = ops.quantise(x.to(cuda_device), fmt_name)
            assert np.array_equal(q.cpu().numpy(), g[f"{name}__q_{fmt_name}"]), f"{name} {fmt_name} bytes"
            assert np.float32(s.item()).view(np.int32) == np.float32(g[f"{name}__s_{fmt_name}"]).view(np.int32)


def _ref_module():
    from oracle import build_ref
    try:
        return build_ref.load()
    except ImportError as e:
        pytest.skip(str(e))


@pytest.mark.parametrize("name,x", [c for c in CASES if c[1].numel() % 8 == 0],
                         ids=[c[0] for c in CASES if c[1].numel() % 8 == 0])
def test_quantise_matches_live_reference_kernel(cuda_device, name, x):
    """Same input through the reference's own CUDA quantiser (oracle/_ref) and ours."""
    R = _ref_module()
    xd = x.to(cuda_device).contiguous()
    for fmt_name, ref_fn in (("e4m3", R.quantise_e4m3), ("e5m2", R.quantise_e5m2)):
        q_ref, s_ref = ref_fn(xd)
        q, s = ops.quantise(xd, fmt_name)
        assert np.float32(s.item()).view(np.int32) == np.float32(s_ref).view(np.int32), (fmt_name, s.item(), s_ref)
        assert torch.equal(q.cpu(), q_ref.cpu()), f"{fmt_name}: bytes differ from the reference kernel"


# ---- GELU + quantise of the FFN activation

def _check_gelu_quant(y16, q, s):
    """The GPU GELU uses the A&S 7.1.26 erf (|err| <= 1.5e-7), the oracle torch's exact erf: fp16 GELU
    values may differ by one ulp, so fp8 codes may differ by one step for a small fraction of elements,
    and the scale (from the amax of the fp16 GELU values) by one fp16 ulp of the amax."""
    from oracle import gemm as ogemm
    g_ref = ogemm.gelu_f16(y16).numpy()
    s_gpu = np.float32(s.item())
    s_ref = fp8.scale_from_amax(fp8.amax_f16(g_ref), fp8.E4M3)
    assert abs(s_gpu / s_ref - 1.0) <= 2.0 ** -10, (s_gpu, s_ref)
    q_ref = fp8.quantise_with_scale(g_ref, s_gpu, fp8.E4M3)
    q = q.cpu().numpy()
    diff = q != q_ref
    assert diff.mean() <= 5e-3, f"{diff.mean():.4%} of fp8 codes differ"
    a = fp8.decode(q[diff], fp8.E4M3).astype(np.float64)
    b = fp8.decode(q_ref[diff], fp8.E4M3).astype(np.float64)
    assert (np.abs(a - b) <= np.maximum(np.abs(a), np.abs(b)) * 2.0 ** -3 + 2.0 ** -9).all()


@pytest.mark.parametrize("std", [0.05, 1.0, 3.0])
def test_quantise_gelu_matches_oracle(cuda_device, std):
    from oracle import gemm as ogemm
    y = randn_f16((777, 1280), 300, std=std)
    yd = y.to(cuda_device)
    key = torch.tensor([ogemm.order_key_f16(float(y.float().max()))], dtype=torch.int32, device=cuda_device)
    q_fast, s_fast = ops.quantise_gelu(yd, key)
    q_full, s_full = ops.quantise_gelu(yd, None)
    # the amax taken from max(y) is exact, so both paths agree bit for bit
    assert torch.equal(q_fast, q_full) and s_fast.item() == s_full.item()
    _check_gelu_quant(y, q_full, s_full)


def test_quantise_gelu_negative_side_amax(cuda_device):
    """All fc1 outputs <= 0.2: gelu(y_max) < 0.171 may not be the amax (negative side up to 0.17), so the
    kernel must take the full pass even when given the max key."""
    from oracle import gemm as ogemm
    y = (-torch.rand(4096, generator=torch.Generator().manual_seed(5)) * 3 + 0.2).half()
    yd = y.to(cuda_device)
    key = torch.tensor([ogemm.order_key_f16(float(y.float().max()))], dtype=torch.int32, device=cuda_device)
    q, s = ops.quantise_gelu(yd, key)
    _check_gelu_quant(y, q, s)
    g = ogemm.gelu_f16(y).float()
    assert abs(s.item() * 448.0 - g.abs().max().item()) <= 2e-3 * g.abs().max().item()


_GELU_FRESH_SCRIPT = r"""
import sys, torch
sys.path.insert(0, {tests!r})
from conftest import randn_f16
from whisper_blaze_b200 import ops
dev = torch.device("cuda:0")
y = randn_f16((1000, 5120), 301).to(dev)
q1, s1 = ops.quantise_gelu(y, None)  # first launch in this process: the CTAs build the table
q2, s2 = ops.quantise_gelu(y, None)  # CTA 0 of the first launch has published it by now
torch.save((q1.cpu(), s1.cpu(), q2.cpu(), s2.cpu()), {path!r})
"""


def test_quantise_gelu_published_table(cuda_device, tmp_path):
    """The GELU table is evaluated by the first launch on a device, which publishes it for the
    CTAs that come later. The first launch in a fresh process and the next one give the same
    codes and scale, equal to this process's result, and meet the oracle gate."""
    import os
    import subprocess
    import sys
    path = str(tmp_path / "gelu_fresh.pt")
    script = _GELU_FRESH_SCRIPT.format(tests=os.path.dirname(os.path.abspath(__file__)), path=path)
    subprocess.run([sys.executable, "-c", script], check=True, timeout=600)
    q1, s1, q2, s2 = torch.load(path)
    assert torch.equal(q1, q2) and torch.equal(s1, s2)
    y = randn_f16((1000, 5120), 301)
    q, s = ops.quantise_gelu(y.to(cuda_device), None)
    assert torch.equal(q.cpu(), q1) and torch.equal(s.cpu(), s1)
    _check_gelu_quant(y, q, s)


@pytest.mark.parametrize("n", [1, 8, 4099, 8192, 81920, 81928, 262144, 262145])
def test_small_tensor_path_matches_two_kernel_path(cuda_device, n):
    """wbk_quantise_f16 takes a single-CTA path up to 262144 elements (register-resident up to 81920,
    n % 8 == 0); it must give the bytes and scale of the amax kernel + quantise kernel pair."""
    x = randn_f16((n,), 400 + n % 97, std=3.0).to(cuda_device)
    q, s = ops.quantise(x)
    ws = ops.new_amax_ws(cuda_device)
    ops.amax_accumulate(x, ws)
    q2, s2 = ops.quantise_from_amax(x, ws)
    assert torch.equal(q, q2) and s.view(torch.int32).item() == s2.view(torch.int32).item()


def _pair_path(x, fmt_name):
    ws = ops.new_amax_ws(x.device)
    ops.amax_accumulate(x, ws)
    q, s = ops.quantise_from_amax(x, ws, fmt_name)
    return q, s, ws


# n from the resident path's lower bound (2^22; every CTA's slice fits in shared memory) past
# the points where the slices outgrow shared memory (148 x 14336 vectors = 17.0M elements) and
# then tensor memory too (148 x 30720 vectors = 36.4M elements) to the 48000 x 1280
# cross-attention input, plus sizes that do not divide evenly among the CTAs.
RESIDENT_SIZES = [1 << 22, (1 << 22) + 8, 16_973_824 + 8 * 1001, 30_000_008, 36_372_480 + 8 * 77, 48000 * 1280]


@pytest.mark.parametrize("fmt_name", ["e4m3", "e5m2"])
@pytest.mark.parametrize("n", RESIDENT_SIZES)
def test_resident_quantise_matches_two_kernel_path(cuda_device, n, fmt_name):
    """wbk_quantise_f16_resident (one cooperative launch, tail of each slice kept on chip)
    gives the codes, scale and amax bits of the amax kernel + quantise kernel pair, and leaves
    its sync words zeroed (checked by running it twice on the same words)."""
    assert n >= ops.RESIDENT_QUANT_MIN
    x = randn_f16((n,), 500 + n % 89, std=2.0).to(cuda_device)
    # the largest magnitude in the last vector (kept on chip) on one run, in the first on another
    sync = torch.zeros(4, dtype=torch.int32, device=cuda_device)
    for pos in (n - 3, 5):
        x[pos] = 3000.0 if pos > 5 else -3500.0
        amax = ops.new_amax_ws(cuda_device)
        q, s = ops.quantise(x, fmt_name, amax_ws=amax, sync_ws=sync)
        q2, s2, ws2 = _pair_path(x, fmt_name)
        assert torch.equal(sync, torch.zeros_like(sync)), "sync words not reset"
        assert amax.item() == ws2.item()
        assert s.view(torch.int32).item() == s2.view(torch.int32).item()
        assert torch.equal(q, q2), f"{int((q != q2).sum())} bytes differ"


@pytest.mark.parametrize("with_inf", [True, False], ids=["inf_amax", "finite_amax"])
@pytest.mark.parametrize("n", [30_000_008, 48000 * 1280])
def test_resident_quantise_specials_and_shared_workspace(cuda_device, n, with_inf):
    """NaN / inf / signed zero anywhere in the slices (shared-memory and TMEM parts, re-read
    front) follow the element rule, with an infinite amax (scale inf, inv 0) and with NaNs but a
    finite amax; the default sync words (the device's shared workspace) work call after call."""
    x = randn_f16((n,), 611, std=1.0).to(cuda_device)
    specials = _special_values(4096, seed=9)
    if not with_inf:
        specials = torch.nan_to_num(specials, nan=float("nan"), posinf=0.0, neginf=0.0)
    specials = specials.to(cuda_device)
    for off in (0, n // 2 - 2048, n - 4096, 21_000_000, n // 3 + 8):
        x[off:off + 4096] = specials
    for _ in range(2):
        q, s = ops.quantise(x)
        q2, s2, _ = _pair_path(x, "e4m3")
        assert s.view(torch.int32).item() == s2.view(torch.int32).item()
        assert torch.equal(q, q2)
    for lo in (0, n // 3, n - 8192):  # against the oracle's element rule, specials included
        q_ref = fp8.quantise_with_scale(x[lo:lo + 8192].cpu().numpy(), np.float32(s.item()), fp8.E4M3)
        assert np.array_equal(q[lo:lo + 8192].cpu().numpy(), q_ref)


@pytest.mark.parametrize("case", ["misaligned_x", "ragged_n", "null_sync", "above_max"])
def test_resident_quantise_falls_back(cuda_device, case):
    """Inputs the resident kernel does not take (x not 16-byte aligned, n % 8 != 0, no sync
    words, more elements than it pays off for) go through wbk_quantise_f16 with the same results."""
    n = ops.RESIDENT_QUANT_MIN + (3 if case == "ragged_n" else 0)
    if case == "above_max":
        n = ops.RESIDENT_QUANT_MAX + 8
    base = randn_f16((n + 8,), 733, std=2.0).to(cuda_device)
    x = base[4:4 + n] if case == "misaligned_x" else base[:n]
    q = torch.empty(n, dtype=torch.uint8, device=cuda_device)
    s = torch.empty(1, dtype=torch.float32, device=cuda_device)
    amax = ops.new_amax_ws(cuda_device)
    sync = torch.zeros(4, dtype=torch.int32, device=cuda_device)
    rc = _lib.lib().wbk_quantise_f16_resident(x.data_ptr(), n, fp8.E4M3, q.data_ptr(), s.data_ptr(),
                                              amax.data_ptr(), 0 if case == "null_sync" else sync.data_ptr(),
                                              torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    q2, s2, ws2 = _pair_path(x, "e4m3")
    assert amax.item() == ws2.item() and torch.equal(q, q2)
    assert s.view(torch.int32).item() == s2.view(torch.int32).item()
