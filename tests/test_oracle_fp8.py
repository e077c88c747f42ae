"""CPU checks of the quantiser oracle (no GPU).

Pins oracle/fp8.py (a) against torch's own float8 casts over every fp16
value, (b) against the reference's own quantiser tests restated
(tests/test_kernels.py:42-79 of whisper-blaze), and (c) against golden
fixtures produced by the reference's CUDA quantiser (tests/golden/).
"""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN_DIR, randn_f16
from oracle import fp8

ALL_F16 = np.arange(65536, dtype=np.uint16).view(np.float16)
FINITE_F16 = ALL_F16[np.isfinite(ALL_F16.astype(np.float32))]


@pytest.mark.parametrize("fmt,tdt", [(fp8.E4M3, torch.float8_e4m3fn), (fp8.E5M2, torch.float8_e5m2)])
@pytest.mark.parametrize("scale", [1.0, 0.37, 3.1e-3, 1e-5, 146.0])
def test_encoder_matches_torch_cast(fmt, tdt, scale):
    mx = fp8.FMT_MAX[fmt]
    v = np.clip(FINITE_F16.astype(np.float32) * np.float32(scale), -mx, mx).astype(np.float32)
    mine = fp8.encode_rne_satfinite(v, fmt)
    ref = torch.from_numpy(v).to(tdt).view(torch.uint8).numpy()
    assert np.array_equal(mine, ref)


@pytest.mark.parametrize("fmt,tdt", [(fp8.E4M3, torch.float8_e4m3fn), (fp8.E5M2, torch.float8_e5m2)])
def test_decode_matches_torch(fmt, tdt):
    codes = torch.arange(256, dtype=torch.uint8)
    tv = codes.view(tdt).float().numpy()
    dv = fp8.decode(codes.numpy(), fmt)
    assert np.array_equal(np.isnan(tv), np.isnan(dv))
    assert np.array_equal(tv[~np.isnan(tv)], dv[~np.isnan(dv)])


def test_known_e4m3_codes():
    # torch's CPU cast, probed: [0.1, 1.0, 447.9, 448, -3.3e-3, 1e-9] -> [29, 56, 126, 126, 130, 0]
    v = np.array([0.1, 1.0, 447.9, 448.0, -3.3e-3, 1e-9], dtype=np.float32)
    assert fp8.encode_rne_satfinite(v, fp8.E4M3).tolist() == [29, 56, 126, 126, 130, 0]


def test_nan_and_inf_semantics():
    # fmaxf(NaN, -448) = -448 in the reference clamp; inf * inv stays inf -> clamp to max
    x = np.array([np.nan, np.inf, -np.inf, 1.0, -0.0, 0.0], dtype=np.float16)
    q = fp8.quantise_with_scale(x, 1.0, fp8.E4M3)
    assert q.tolist() == [0xFE, 0x7E, 0xFE, 56, 0x80, 0x00]
    # amax ignores NaN; inf amax -> scale inf -> inv 0 -> finite * 0 = 0, inf * 0 = NaN -> -448
    assert fp8.amax_f16(x) == np.inf
    q2, s2 = fp8.quantise(x, fp8.E4M3)
    assert s2 == np.inf
    assert q2.tolist() == [0xFE, 0xFE, 0xFE, 0x00, 0x80, 0x00]


def test_all_nan_or_empty_gives_scale_one():
    assert fp8.quantise(np.full(16, np.nan, dtype=np.float16))[1] == 1.0
    assert fp8.quantise(np.zeros(0, dtype=np.float16))[1] == 1.0


# ---- the reference's own quantiser tests (tests/test_kernels.py:42-79), restated on the oracle

def _round_trip(x16, fmt):
    q, s = fp8.quantise(x16.numpy(), fmt)
    return torch.from_numpy(fp8.dequantise(q, s, fmt)), s, q


def test_ref_e4m3_roundtrip_shape():
    x = randn_f16((128, 512), 1)
    q, _ = fp8.quantise(x.numpy(), fp8.E4M3)
    assert q.shape == tuple(x.shape)


def test_ref_e4m3_roundtrip_values():
    x = randn_f16((512, 512), 2)
    xh, _, _ = _round_trip(x, fp8.E4M3)
    assert torch.allclose(x.float(), xh.float(), atol=0.1, rtol=0.2)


def test_ref_e5m2_roundtrip_values():
    x = randn_f16((512, 512), 3)
    xh, _, _ = _round_trip(x, fp8.E5M2)
    assert torch.allclose(x.float(), xh.float(), atol=0.2, rtol=0.3)


def test_ref_scale_positive():
    x = randn_f16((256, 256), 4)
    assert fp8.quantise(x.numpy(), fp8.E4M3)[1] > 0
    assert fp8.quantise(x.numpy(), fp8.E5M2)[1] > 0


def test_ref_zero_tensor():
    x = torch.zeros(64, 64, dtype=torch.float16)
    xh, s, _ = _round_trip(x, fp8.E4M3)
    assert s == 1.0
    assert torch.allclose(xh.float(), x.float(), atol=1e-6)


# ---- golden fixtures from the reference's CUDA quantiser (generated on a B200)

GOLDEN_QUANT = os.path.join(GOLDEN_DIR, "ref_quantise.npz")
GOLDEN_SCALES = os.path.join(GOLDEN_DIR, "ref_scale_table.npz")


def _require(path):
    if not os.path.exists(path):
        pytest.fail(f"golden fixture {path} is missing (generate with tests/golden/make_golden.py on a B200)")


def test_golden_quantise_bytes_match_oracle():
    """For every golden case, the oracle's element rule reproduces the reference
    kernel's bytes exactly from the reference kernel's own scale."""
    _require(GOLDEN_QUANT)
    g = np.load(GOLDEN_QUANT)
    names = sorted({k.split("__")[0] for k in g.files})
    assert names
    for name in names:
        x = g[f"{name}__x"]
        for fmt_name, fmt in fp8.FMT_NAMES.items():
            q_ref = g[f"{name}__q_{fmt_name}"]
            s_ref = np.float32(g[f"{name}__s_{fmt_name}"])
            q = fp8.quantise_with_scale(x, s_ref, fmt)
            assert np.array_equal(q, q_ref), f"{name} {fmt_name}: {np.count_nonzero(q != q_ref)} bytes differ"
            # dequantise is exact given the same bytes and scale (NaN payloads aside)
            dq_ref = g[f"{name}__dq_{fmt_name}"]
            dq = fp8.dequantise(q_ref, s_ref, fmt)
            nan = np.isnan(dq_ref.astype(np.float32))
            assert np.array_equal(np.isnan(dq.astype(np.float32)), nan)
            assert np.array_equal(dq[~nan].view(np.uint16), dq_ref[~nan].view(np.uint16))


def test_golden_scale_table_vs_ieee():
    """The reference computes amax/max_fp8 with the fast-math division. For every
    positive finite fp16 amax, its scale is within 1 ulp of the IEEE quotient
    the oracle uses; the count of inputs where they differ is reported."""
    _require(GOLDEN_SCALES)
    g = np.load(GOLDEN_SCALES)
    amax = g["amax_bits"].view(np.float16).astype(np.float32)
    for fmt_name, fmt in fp8.FMT_NAMES.items():
        ref = g[f"scale_{fmt_name}"].astype(np.float32)
        ieee = np.array([fp8.scale_from_amax(a, fmt) for a in amax], dtype=np.float32)
        ulp = np.abs(ref.view(np.int32).astype(np.int64) - ieee.view(np.int32).astype(np.int64))
        assert ulp.max() <= 1, f"{fmt_name}: fast-math scale differs from IEEE by {ulp.max()} ulp"
        print(f"{fmt_name}: {np.count_nonzero(ulp)} of {len(amax)} amax values differ from IEEE by 1 ulp")
