"""Tensor-level wrappers over libwbk.so for torch callers.

Every op runs on torch's current stream of its input's device, under a device
guard, and never synchronises unless it must hand a value back to the host.
Scales can stay on the device (1-element fp32 tensors), so a chain of
quantise -> GEMM -> norm -> quantise issues no host round trip.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Sequence, Union

import torch

from . import _lib
from ._lib import (EPI_BIAS_MAXKEY, EPI_GELU, EPI_NONE, EPI_RESIDUAL, EPI_RESIDUAL_CLAMP, FMT_E4M3, FMT_E5M2,
                   check, lib, ptr, stream_of)

Scale = Union[float, torch.Tensor]

# Number of libwbk kernels launched by this process (quantise() launches the
# amax and the quantise kernel, 2; every other op launches 1).
LAUNCHES = [0]


def _count(n: int = 1) -> None:
    LAUNCHES[0] += n


_FMT_BY_NAME = {"e4m3": FMT_E4M3, "e5m2": FMT_E5M2, FMT_E4M3: FMT_E4M3, FMT_E5M2: FMT_E5M2}
_EPI_BY_NAME = {"none": EPI_NONE, "bias": EPI_NONE, "gelu": EPI_GELU, "residual": EPI_RESIDUAL,
                "residual_clamp": EPI_RESIDUAL_CLAMP, "bias_maxkey": EPI_BIAS_MAXKEY, EPI_NONE: EPI_NONE,
                EPI_GELU: EPI_GELU, EPI_RESIDUAL: EPI_RESIDUAL, EPI_RESIDUAL_CLAMP: EPI_RESIDUAL_CLAMP,
                EPI_BIAS_MAXKEY: EPI_BIAS_MAXKEY}
_BYTE_DTYPES = {torch.uint8, torch.int8, torch.float8_e4m3fn, torch.float8_e5m2}


def fmt_code(fmt) -> int:
    try:
        return _FMT_BY_NAME[fmt]
    except KeyError:
        raise ValueError(f"unknown fp8 format {fmt!r}; expected 'e4m3' or 'e5m2'") from None


def require_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")


def require_contig(t: torch.Tensor, name: str) -> None:
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def require_input(t: torch.Tensor, name: str) -> None:
    require_cuda(t, name)
    require_contig(t, name)


def require_fp16(t: torch.Tensor, name: str) -> None:
    if t.dtype != torch.float16:
        raise RuntimeError(f"{name} must be fp16")


def require_bytes(t: torch.Tensor, name: str) -> None:
    if t.dtype not in _BYTE_DTYPES:
        raise RuntimeError(f"{name} must hold fp8 codes (uint8 or a float8 dtype), got {t.dtype}")


def require_same_device(*ts: Optional[torch.Tensor]) -> None:
    devs = {t.device for t in ts if t is not None}
    if len(devs) > 1:
        raise RuntimeError(f"tensors are on different devices: {sorted(map(str, devs))}")


def new_amax_ws(device) -> torch.Tensor:
    """A zeroed device uint32 accumulator (held as int32) for the fused amax."""
    return torch.zeros(1, dtype=torch.int32, device=device)


# ---------------------------------------------------------------- quantiser

def amax_accumulate(x: torch.Tensor, amax_ws: torch.Tensor) -> torch.Tensor:
    require_input(x, "x")
    require_fp16(x, "x")
    require_same_device(x, amax_ws)
    with torch.cuda.device(x.device):
        check(lib().wbk_amax_f16(x.data_ptr(), x.numel(), amax_ws.data_ptr(), stream_of(x)), "amax")
    _count()
    return amax_ws


def quantise_from_amax(x: torch.Tensor, amax_ws: torch.Tensor, fmt="e4m3", q_out: Optional[torch.Tensor] = None,
                       scale_out: Optional[torch.Tensor] = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Quantise x with the scale implied by an already accumulated amax."""
    require_input(x, "x")
    require_fp16(x, "x")
    f = fmt_code(fmt)
    q = torch.empty(x.shape, dtype=torch.uint8, device=x.device) if q_out is None else q_out
    s = torch.empty(1, dtype=torch.float32, device=x.device) if scale_out is None else scale_out
    require_same_device(x, amax_ws, q, s)
    with torch.cuda.device(x.device):
        check(lib().wbk_quantise_from_amax_f16(x.data_ptr(), x.numel(), f, amax_ws.data_ptr(), q.data_ptr(),
                                               s.data_ptr(), stream_of(x)), "quantise")
    _count()
    return q, s


# Tensors of RESIDENT_QUANT_MIN to RESIDENT_QUANT_MAX elements (a multiple of 8,
# 16-byte aligned) are quantised by the one-launch resident kernel
# (wbk_quantise_f16_resident); the library applies the same bounds.
RESIDENT_QUANT_MIN = 1 << 22
RESIDENT_QUANT_MAX = 88 << 20
_RESIDENT_SYNC_OFFSET = 32  # bytes: words 8..11 of the device's shared workspace (the GEMM's use 0..3)


def quantise(x: torch.Tensor, fmt="e4m3", q_out: Optional[torch.Tensor] = None,
             scale_out: Optional[torch.Tensor] = None,
             amax_ws: Optional[torch.Tensor] = None,
             sync_ws: Optional[torch.Tensor] = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-tensor quantise; returns (codes uint8, device fp32 scale [1]). No host sync.

    Large tensors (RESIDENT_QUANT_MIN to RESIDENT_QUANT_MAX elements) take one cooperative
    launch that reads x from HBM about once; its grid-wide arrival uses 16 bytes
    of sync words, by default in the device's shared workspace, so such calls
    must not run concurrently on different streams: pass `sync_ws` (a zeroed
    device tensor of 16 bytes, left zeroed by each call) to give a stream its
    own. Codes, scale and amax are the same on either path."""
    require_input(x, "x")
    require_fp16(x, "x")
    f = fmt_code(fmt)
    q = torch.empty(x.shape, dtype=torch.uint8, device=x.device) if q_out is None else q_out
    s = torch.empty(1, dtype=torch.float32, device=x.device) if scale_out is None else scale_out
    ws = torch.empty(1, dtype=torch.int32, device=x.device) if amax_ws is None else amax_ws
    require_same_device(x, q, s, ws, sync_ws)
    n = x.numel()
    with torch.cuda.device(x.device):
        if (RESIDENT_QUANT_MIN <= n <= RESIDENT_QUANT_MAX and n % 8 == 0 and x.data_ptr() % 16 == 0
                and q.data_ptr() % 8 == 0):
            if sync_ws is None:
                sync_ptr = splitk_workspace(x.device, 256).data_ptr() + _RESIDENT_SYNC_OFFSET
            else:
                if sync_ws.numel() * sync_ws.element_size() < 16 or sync_ws.data_ptr() % 16 != 0:
                    raise ValueError("sync_ws must hold 16 bytes at a 16-byte aligned address")
                sync_ptr = sync_ws.data_ptr()
            check(lib().wbk_quantise_f16_resident(x.data_ptr(), n, f, q.data_ptr(), s.data_ptr(), ws.data_ptr(),
                                                  sync_ptr, stream_of(x)), "quantise")
            _count(1)
        else:
            check(lib().wbk_quantise_f16(x.data_ptr(), n, f, q.data_ptr(), s.data_ptr(), ws.data_ptr(),
                                         stream_of(x)), "quantise")
            _count(2)
    return q, s


def quantise_gelu(y: torch.Tensor, ymax_key: Optional[torch.Tensor] = None, fmt="e4m3",
                  q_out: Optional[torch.Tensor] = None, scale_out: Optional[torch.Tensor] = None,
                  amax_ws: Optional[torch.Tensor] = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Quantise fp16(gelu(y)) per tensor without storing the GELU output.

    ymax_key: the max-key word written by a GEMM with the 'bias_maxkey'
    epilogue over y (lets the amax come from y's maximum), or None."""
    require_input(y, "y")
    require_fp16(y, "y")
    f = fmt_code(fmt)
    q = torch.empty(y.shape, dtype=torch.uint8, device=y.device) if q_out is None else q_out
    s = torch.empty(1, dtype=torch.float32, device=y.device) if scale_out is None else scale_out
    ws = torch.empty(1, dtype=torch.int32, device=y.device) if amax_ws is None else amax_ws
    require_same_device(y, ymax_key, q, s, ws)
    with torch.cuda.device(y.device):
        check(lib().wbk_quantise_gelu_f16(y.data_ptr(), y.numel(), f, ptr(ymax_key), q.data_ptr(), s.data_ptr(),
                                          ws.data_ptr(), stream_of(y)), "quantise_gelu")
    _count(2)
    return q, s


def dequantise(q: torch.Tensor, scale: float, shape: Sequence[int], fmt="e4m3") -> torch.Tensor:
    require_input(q, "fp8")
    require_bytes(q, "fp8")
    f = fmt_code(fmt)
    shape = [int(d) for d in shape]
    out = torch.empty(shape, dtype=torch.float16, device=q.device)
    if out.numel() != q.numel():
        raise RuntimeError(f"shape {shape} holds {out.numel()} elements but fp8 has {q.numel()}")
    with torch.cuda.device(q.device):
        check(lib().wbk_dequantise_f16(q.data_ptr(), q.numel(), f, float(scale), out.data_ptr(), stream_of(q)),
              "dequantise")
    _count()
    return out


# -------------------------------------------------------------------- norms

def layernorm(x: torch.Tensor, residual: Optional[torch.Tensor], gamma: torch.Tensor, beta: torch.Tensor,
              eps: float = 1e-5, want_sum: bool = False, out: Optional[torch.Tensor] = None,
              sum_out: Optional[torch.Tensor] = None,
              out_amax: Optional[torch.Tensor] = None) -> tuple[torch.Tensor, Optional[torch.Tensor]]:
    require_input(x, "x")
    require_input(gamma, "gamma")
    require_input(beta, "beta")
    require_fp16(x, "x")
    require_fp16(gamma, "gamma")
    require_fp16(beta, "beta")
    if residual is not None:
        require_input(residual, "residual")
        require_fp16(residual, "residual")
        if residual.shape != x.shape:
            raise RuntimeError("residual must have the same shape as x")
    if x.dim() == 0:
        raise RuntimeError("x must have at least one dimension")
    D = x.shape[-1]
    if gamma.numel() != D or beta.numel() != D:
        raise RuntimeError(f"gamma and beta must have {D} elements")
    rows = x.numel() // D if D else 0
    o = torch.empty_like(x) if out is None else out
    s = (torch.empty_like(x) if sum_out is None else sum_out) if want_sum else None
    require_same_device(x, residual, gamma, beta, o, s, out_amax)
    with torch.cuda.device(x.device):
        check(lib().wbk_layernorm_f16(x.data_ptr(), ptr(residual), gamma.data_ptr(), beta.data_ptr(), o.data_ptr(),
                                      ptr(s), rows, D, float(eps), ptr(out_amax), stream_of(x)), "layernorm_fused")
    _count()
    return o, s


def layernorm_quantise_ws(rows: int, device) -> torch.Tensor:
    """Workspace for layernorm_quantise: per-row statistics + the (scale, 1/scale) pair."""
    return torch.empty(int(lib().wbk_layernorm_quantise_ws_bytes(int(rows))), dtype=torch.uint8, device=device)


def layernorm_quantise(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, eps: float = 1e-5, fmt="e4m3",
                       q_out: Optional[torch.Tensor] = None, scale_out: Optional[torch.Tensor] = None,
                       ws: Optional[torch.Tensor] = None,
                       amax_ws: Optional[torch.Tensor] = None) -> tuple[torch.Tensor, torch.Tensor]:
    """fp8 codes of LayerNorm(x) (no residual), bit-identical to layernorm() then quantise(),
    without writing the fp16 LayerNorm output."""
    require_input(x, "x")
    require_input(gamma, "gamma")
    require_input(beta, "beta")
    require_fp16(x, "x")
    require_fp16(gamma, "gamma")
    require_fp16(beta, "beta")
    D = x.shape[-1]
    if gamma.numel() != D or beta.numel() != D:
        raise RuntimeError(f"gamma and beta must have {D} elements")
    rows = x.numel() // D if D else 0
    f = fmt_code(fmt)
    q = torch.empty(x.shape, dtype=torch.uint8, device=x.device) if q_out is None else q_out
    s = torch.empty(1, dtype=torch.float32, device=x.device) if scale_out is None else scale_out
    w = layernorm_quantise_ws(rows, x.device) if ws is None else ws
    a = torch.empty(1, dtype=torch.int32, device=x.device) if amax_ws is None else amax_ws
    if w.numel() < lib().wbk_layernorm_quantise_ws_bytes(rows):
        raise RuntimeError("layernorm_quantise workspace too small")
    require_same_device(x, gamma, beta, q, s, w, a)
    with torch.cuda.device(x.device):
        check(lib().wbk_layernorm_quantise_f16(x.data_ptr(), gamma.data_ptr(), beta.data_ptr(), rows, D, float(eps), f,
                                               q.data_ptr(), s.data_ptr(), w.data_ptr(), a.data_ptr(), stream_of(x)),
              "layernorm_quantise")
    _count(2)
    return q, s


def rmsnorm(x: torch.Tensor, residual: torch.Tensor, gamma: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    require_input(x, "x")
    require_input(residual, "residual")
    require_input(gamma, "gamma")
    require_fp16(x, "x")
    require_fp16(residual, "residual")
    require_fp16(gamma, "gamma")
    if residual.shape != x.shape:
        raise RuntimeError("residual must have the same shape as x")
    D = x.shape[-1]
    if gamma.numel() != D:
        raise RuntimeError(f"gamma must have {D} elements")
    out = torch.empty_like(x)
    require_same_device(x, residual, gamma)
    with torch.cuda.device(x.device):
        check(lib().wbk_rmsnorm_f16(x.data_ptr(), residual.data_ptr(), gamma.data_ptr(), out.data_ptr(),
                                    x.numel() // D, D, float(eps), stream_of(x)), "rmsnorm_fused")
    _count()
    return out


# --------------------------------------------------------------------- GEMM

def _scale_arg(scale: Scale, name: str, device) -> tuple[float, Optional[int]]:
    if isinstance(scale, torch.Tensor):
        if scale.numel() != 1 or scale.dtype != torch.float32 or not scale.is_cuda:
            raise RuntimeError(f"{name} must be a Python float or a 1-element fp32 CUDA tensor")
        if scale.device != device:
            raise RuntimeError(f"{name} is on {scale.device}, expected {device}")
        return 1.0, scale.data_ptr()
    return float(scale), None


_SPLITK_WS: dict = {}


@_lib.on_device_timeout
def _zero_shared_workspaces(device_index: int) -> None:
    """After a device-side timeout a kernel may have left the sync words or split-K tickets of
    the device's shared workspace non-zero; zero it again so the next call starts clean.
    (Workspaces passed by the caller are the caller's to zero, as wbk.h states.)"""
    ws = _SPLITK_WS.get(torch.device("cuda", device_index))
    if ws is not None:
        ws.zero_()


def splitk_workspace(device, nbytes: int) -> Optional[torch.Tensor]:
    """The per-device split-K workspace (zero-filled once, grown on demand).

    Shared by every short-M GEMM on the device, so such GEMMs must not run
    concurrently on different streams; pass `workspace=` to gemm_fp8 to give a
    stream its own."""
    if nbytes <= 0:
        return None
    dev = torch.device(device)
    ws = _SPLITK_WS.get(dev)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        _SPLITK_WS[dev] = ws
    return ws


def _check_epilogue_args(epilogue, M: int, N: int, out_shape, bias, residual, out_amax) -> int:
    epi = _EPI_BY_NAME.get(epilogue)
    if epi is None:
        raise ValueError(f"unknown epilogue {epilogue!r}")
    if bias is not None:
        require_input(bias, "bias")
        require_fp16(bias, "bias")
        if bias.numel() != N:
            raise RuntimeError(f"bias must have {N} elements")
    if residual is not None:
        require_input(residual, "residual")
        require_fp16(residual, "residual")
        if residual.numel() != M * N:
            raise RuntimeError(f"residual must have shape {out_shape}")
    if epi in (EPI_RESIDUAL, EPI_RESIDUAL_CLAMP) and residual is None:
        raise RuntimeError("residual epilogue requires a residual tensor")
    if epi == EPI_BIAS_MAXKEY and out_amax is None:
        raise RuntimeError("the bias_maxkey epilogue requires out_amax")
    return epi


def gemm_fp8(a: torch.Tensor, a_scale: Scale, w: torch.Tensor, w_scale: Scale,
             bias: Optional[torch.Tensor] = None, residual: Optional[torch.Tensor] = None, epilogue="none",
             a_format="e4m3", w_format="e4m3", out: Optional[torch.Tensor] = None,
             out_amax: Optional[torch.Tensor] = None, workspace: Optional[torch.Tensor] = None,
             split_k: bool = True) -> torch.Tensor:
    """out[..., N] = epilogue(dq(a)[..., K] @ dq(w)[N, K]^T + bias); fp16 output.

    a: fp8 codes [..., K]; w: fp8 codes [N, K] (nn.Linear layout); scales as
    Python floats or 1-element fp32 CUDA tensors; epilogue one of
    'none' | 'gelu' | 'residual' | 'residual_clamp' | 'bias_maxkey' (bias only, and
    out_amax receives the order key of the largest output, for quantise_gelu).
    Short-M shapes (M <= 128) split K over more SMs (split_k=True) using
    `workspace` (a zero-filled uint8 CUDA tensor of at least
    wbk_gemm_fp8_ws_bytes bytes) or the device's shared one.
    """
    require_input(a, "a_fp8")
    require_input(w, "w_fp8")
    require_bytes(a, "a_fp8")
    require_bytes(w, "w_fp8")
    if w.dim() != 2:
        raise RuntimeError("w_fp8 must be 2-D [N, K]")
    N, K = w.shape
    if a.dim() < 1 or a.shape[-1] != K:
        raise RuntimeError(f"a_fp8 last dimension {a.shape[-1] if a.dim() else None} != K={K}")
    M = a.numel() // K if K else 0
    out_shape = tuple(a.shape[:-1]) + (N,)
    epi = _check_epilogue_args(epilogue, M, N, out_shape, bias, residual, out_amax)
    alpha_a, pa = _scale_arg(a_scale, "a_scale", a.device)
    alpha_w, pw = _scale_arg(w_scale, "w_scale", a.device)
    alpha = float(torch.tensor(alpha_a, dtype=torch.float32) * torch.tensor(alpha_w, dtype=torch.float32))
    o = torch.empty(out_shape, dtype=torch.float16, device=a.device) if out is None else out
    require_same_device(a, w, bias, residual, o, out_amax, workspace)
    with torch.cuda.device(a.device):
        ws = None
        if split_k and 0 < M <= 128:
            need = lib().wbk_gemm_fp8_ws_bytes(M, N, K)
            ws = workspace if workspace is not None else splitk_workspace(a.device, need)
        check(lib().wbk_gemm_fp8_ws(a.data_ptr(), w.data_ptr(), M, N, K, fmt_code(a_format), fmt_code(w_format),
                                    alpha, pa, pw, ptr(bias), ptr(residual), o.data_ptr(), epi, ptr(out_amax),
                                    ptr(ws), 0 if ws is None else ws.numel(), stream_of(a)),
              "gemm_fp8")
    _count()
    return o


def linear_fp8(x: torch.Tensor, w: torch.Tensor, w_scale: Scale, bias: Optional[torch.Tensor] = None,
               residual: Optional[torch.Tensor] = None, epilogue="none", a_format="e4m3", w_format="e4m3",
               out: Optional[torch.Tensor] = None, out_amax: Optional[torch.Tensor] = None,
               q_out: Optional[torch.Tensor] = None, scale_out: Optional[torch.Tensor] = None,
               amax_ws: Optional[torch.Tensor] = None,
               workspace: Optional[torch.Tensor] = None) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """FP8 linear on an fp16 activation: quantise(x) then gemm_fp8, as one call.

    x: fp16 [..., K]; w: fp8 codes [N, K]. Returns (out fp16 [..., N], x's codes
    uint8 [..., K], x's scale fp32 [1]) -- the codes and scale are exactly what
    quantise(x) returns, the output exactly gemm_fp8 of them. For M <= 128 rows
    this is one kernel (the GEMM quantises x itself) using `workspace` or the
    device's shared one; otherwise the quantiser kernel and the GEMM.
    """
    require_input(x, "x")
    require_fp16(x, "x")
    require_input(w, "w_fp8")
    require_bytes(w, "w_fp8")
    if w.dim() != 2:
        raise RuntimeError("w_fp8 must be 2-D [N, K]")
    N, K = w.shape
    if x.dim() < 1 or x.shape[-1] != K:
        raise RuntimeError(f"x last dimension {x.shape[-1] if x.dim() else None} != K={K}")
    M = x.numel() // K if K else 0
    out_shape = tuple(x.shape[:-1]) + (N,)
    epi = _check_epilogue_args(epilogue, M, N, out_shape, bias, residual, out_amax)
    alpha, pw = _scale_arg(w_scale, "w_scale", x.device)
    q = torch.empty(x.shape, dtype=torch.uint8, device=x.device) if q_out is None else q_out
    sc = torch.empty(1, dtype=torch.float32, device=x.device) if scale_out is None else scale_out
    aws = torch.empty(1, dtype=torch.int32, device=x.device) if amax_ws is None else amax_ws
    o = torch.empty(out_shape, dtype=torch.float16, device=x.device) if out is None else out
    require_same_device(x, w, bias, residual, o, out_amax, q, sc, aws, workspace)
    with torch.cuda.device(x.device):
        ws = None
        if 0 < M <= 128:
            need = lib().wbk_gemm_fp8_ws_bytes(M, N, K)
            ws = workspace if workspace is not None else splitk_workspace(x.device, need)
        check(lib().wbk_linear_fp8_f16(x.data_ptr(), M, N, K, fmt_code(a_format), q.data_ptr(), sc.data_ptr(),
                                       aws.data_ptr(), w.data_ptr(), fmt_code(w_format), pw, alpha, ptr(bias),
                                       ptr(residual), o.data_ptr(), epi, ptr(out_amax), ptr(ws),
                                       0 if ws is None else ws.numel(), stream_of(x)),
              "linear_fp8")
    _count(1 if 0 < M <= 128 else 2)
    return o, q, sc


# ---------------------------------------------------------------- attention

def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: Optional[torch.Tensor] = None,
              scale: Optional[float] = None, out_amax: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Non-causal attention, head dim 64: softmax(q k^T * scale) v.

    q [B, H, Sq, 64], k and v [B, H, Sk, 64] fp16 CUDA views (any strides that
    are multiples of 8 elements, last dimension contiguous), e.g. the q/k/v
    slices of a fused QKV projection; `out` likewise (default: a new contiguous
    [B, H, Sq, 64] tensor). scale defaults to 1/sqrt(64). out_amax (optional, an
    amax workspace) max-accumulates max|out|.
    """
    for t, name in ((q, "Q"), (k, "K"), (v, "V")):
        require_cuda(t, name)
        require_fp16(t, name)
        if t.dim() != 4:
            raise RuntimeError(f"{name} must be 4D: [B, H, S, D]")
        if t.stride(-1) != 1:
            raise RuntimeError(f"{name} must have a contiguous last dimension")
    B, H, Sq, D = q.shape
    if k.shape[:2] != (B, H) or v.shape[:2] != (B, H) or k.shape[-1] != D or v.shape[-1] != D:
        raise RuntimeError("Q, K and V must agree in batch, heads and head dim")
    if k.shape[2] != v.shape[2]:
        raise RuntimeError("K and V must have the same sequence length")
    Sk = k.shape[2]
    o = torch.empty((B, H, Sq, D), dtype=torch.float16, device=q.device) if out is None else out
    if o.shape != (B, H, Sq, D) or o.dtype != torch.float16 or o.stride(-1) != 1:
        raise RuntimeError(f"out must be an fp16 [B, H, Sq, D] = {(B, H, Sq, D)} view with a contiguous last dimension")
    require_same_device(q, k, v, o, out_amax)
    strides = (ctypes.c_int64 * 12)(*(list(q.stride()[:3]) + list(k.stride()[:3]) + list(v.stride()[:3]) +
                                      list(o.stride()[:3])))
    sc = float(scale) if scale is not None else D ** -0.5
    with torch.cuda.device(q.device):
        check(lib().wbk_attention_f16(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), B, H, Sq, Sk, D,
                                      strides, sc, ptr(out_amax), stream_of(q)), "attention")
    _count()
    return o
