"""CPU restatement of the reference FP8 quantiser (test infrastructure only).

Follows csrc/kernels/fp8_quantize.cu of whisper-blaze v0.1.17:

* amax       — max over elements of fabsf(float(x)); fmaxf ignores NaN
               (compute_scale_kernel, fp8_quantize.cu:54-59);
* scale      — amax / max_fp8 (fp8_quantize.cu:72), replaced by 1.0 unless
               it is > 0 (compute_fp8_scale, :218). The reference evaluates
               the division on the GPU under --use_fast_math; this oracle uses
               the IEEE quotient, and the GPU tests compare the product's scale
               against the reference kernel's own output (tests/golden);
* inv_scale  — 1.0f / scale in IEEE single precision on the host (:224);
* quantise   — q = fp8_rn_satfinite(fminf(fmaxf(float(x)*inv_scale, -max), max))
               (quantise_fp16_to_e4m3_kernel, :99-105); fmaxf/fminf turn a NaN
               product into -max;
* dequantise — fp16(float(q) * scale) (dequantise_e4m3_to_fp16_kernel, :157-159).

The fp8 encoder below is an independent table-based round-to-nearest-even
implementation of the OCP FP8 formats (E4M3FN: bias 7, max 448, S.1111.111 is
NaN; E5M2: bias 15, max 57344, exponent 11111 is Inf/NaN), cross-checked
against torch's float8 casts in tests/test_oracle_fp8.py.
"""
from __future__ import annotations

import numpy as np

E4M3 = 0
E5M2 = 1
FMT_MAX = {E4M3: np.float32(448.0), E5M2: np.float32(57344.0)}
FMT_NAMES = {"e4m3": E4M3, "e5m2": E5M2}


def _decode_table(fmt: int) -> np.ndarray:
    """float32 value of each of the 256 codes of `fmt` (NaN for NaN codes)."""
    ebits, mbits, bias = (4, 3, 7) if fmt == E4M3 else (5, 2, 15)
    out = np.empty(256, dtype=np.float32)
    for code in range(256):
        sign = -1.0 if code & 0x80 else 1.0
        e = (code >> mbits) & ((1 << ebits) - 1)
        m = code & ((1 << mbits) - 1)
        if fmt == E4M3 and e == 0xF and m == 0x7:
            v = np.nan
        elif fmt == E5M2 and e == 0x1F:
            v = sign * np.inf if m == 0 else np.nan
        elif e == 0:
            v = sign * (m / (1 << mbits)) * 2.0 ** (1 - bias)
        else:
            v = sign * (1.0 + m / (1 << mbits)) * 2.0 ** (e - bias)
        if not np.isnan(v) and not np.isinf(v):
            v = sign * abs(v)
        out[code] = v
    return out


_DECODE = {E4M3: _decode_table(E4M3), E5M2: _decode_table(E5M2)}


def _positive_finite(fmt: int) -> tuple[np.ndarray, np.ndarray]:
    """Sorted non-negative finite values and their codes (codes 0x00..max)."""
    table = _DECODE[fmt]
    last = 0x7E if fmt == E4M3 else 0x7B
    codes = np.arange(0, last + 1, dtype=np.int64)
    return table[codes].astype(np.float64), codes


_POS = {E4M3: _positive_finite(E4M3), E5M2: _positive_finite(E5M2)}


def decode(q: np.ndarray, fmt: int) -> np.ndarray:
    """fp8 codes (uint8) -> float32 values (exact)."""
    return _DECODE[fmt][np.asarray(q, dtype=np.uint8)]


def encode_rne_satfinite(v: np.ndarray, fmt: int) -> np.ndarray:
    """float32 -> fp8 code, round to nearest (ties to even), saturate to the
    largest finite value. NaN maps to the format's canonical NaN (0x7F); it
    never occurs on the quantise path because the clamp removes it first."""
    v = np.asarray(v, dtype=np.float32)
    vals, codes = _POS[fmt]
    a = np.abs(v).astype(np.float64)
    sat = np.minimum(a, vals[-1])
    hi = np.clip(np.searchsorted(vals, sat, side="left"), 0, len(vals) - 1)
    lo = np.clip(hi - 1, 0, len(vals) - 1)
    d_lo = sat - vals[lo]
    d_hi = vals[hi] - sat
    pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & (codes[hi] % 2 == 0))
    pick_hi |= hi == lo
    mag = np.where(pick_hi, codes[hi], codes[lo])
    sign = np.signbit(v).astype(np.int64) << 7
    out = (mag | sign).astype(np.uint8)
    out = np.where(np.isnan(v), np.uint8(0x7F), out)
    return out.astype(np.uint8)


def amax_f16(x: np.ndarray) -> np.float32:
    """max |x| over an fp16 array, NaNs ignored, 0 for empty or all-NaN."""
    a = np.abs(np.asarray(x, dtype=np.float16).astype(np.float32)).ravel()
    a = a[~np.isnan(a)]
    return np.float32(a.max()) if a.size else np.float32(0.0)


def scale_from_amax(amax: float, fmt: int) -> np.float32:
    """IEEE amax / max_fp8, or 1.0 unless that is > 0."""
    s = np.float32(amax) / FMT_MAX[fmt]
    return np.float32(s) if s > 0 else np.float32(1.0)


def inv_scale(scale: float) -> np.float32:
    with np.errstate(divide="ignore"):
        return np.float32(np.float32(1.0) / np.float32(scale))


def quantise_with_scale(x: np.ndarray, scale: float, fmt: int) -> np.ndarray:
    """fp16 array -> fp8 codes for a given scale (the kernel's element rule)."""
    mx = FMT_MAX[fmt]
    inv = inv_scale(scale)
    with np.errstate(invalid="ignore", over="ignore"):
        f = np.asarray(x, dtype=np.float16).astype(np.float32) * inv
    c = np.fmin(np.fmax(f, np.float32(-mx)), mx)  # C fmaxf/fminf: NaN -> -mx
    c = np.where(np.isnan(f), -mx, c).astype(np.float32)
    return encode_rne_satfinite(c, fmt)


def quantise(x: np.ndarray, fmt: int = E4M3) -> tuple[np.ndarray, np.float32]:
    """Reference quantise_to_e4m3 / _e5m2: returns (codes, scale)."""
    scale = scale_from_amax(amax_f16(x), fmt)
    return quantise_with_scale(x, scale, fmt), scale


def quantise_torch(x, fmt: int = E4M3):
    """Same rule as quantise(), vectorised on torch-CPU (multi-threaded) for the
    timed CPU path: amax ignoring NaN, IEEE scale, fp32 multiply, NaN -> -max,
    clamp, torch's round-to-nearest-even fp8 cast (bit-identical to
    encode_rne_satfinite on clamped values, see tests/test_oracle_fp8.py).
    Returns (uint8 codes tensor, float32 scale)."""
    import torch
    xf = x.float()
    a = xf.abs()
    a = torch.where(torch.isnan(a), torch.zeros_like(a), a)
    amax = np.float32(a.max().item()) if a.numel() else np.float32(0.0)
    scale = scale_from_amax(amax, fmt)
    inv = float(inv_scale(scale))
    mx = float(FMT_MAX[fmt])
    f = xf * torch.tensor(inv, dtype=torch.float32)
    c = torch.where(torch.isnan(f), torch.full_like(f, -mx), f.clamp(-mx, mx))
    dt = torch.float8_e4m3fn if fmt == E4M3 else torch.float8_e5m2
    return c.to(dt).view(torch.uint8), scale


def dequantise(q: np.ndarray, scale: float, fmt: int = E4M3) -> np.ndarray:
    """Reference dequantise: fp16(float(q) * scale)."""
    with np.errstate(over="ignore", invalid="ignore"):
        return (decode(q, fmt) * np.float32(scale)).astype(np.float16)


def dequantise_f32(q: np.ndarray, scale: float, fmt: int = E4M3) -> np.ndarray:
    """fp32 dequantisation (no fp16 rounding), the GEMM oracle's operand."""
    return decode(q, fmt) * np.float32(scale)
