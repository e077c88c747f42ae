"""ctypes binding of libwbk.so (the C ABI declared in include/wbk.h).

The library is loaded from this source tree (whisper-blaze_b200/lib/libwbk.so);
there is no fallback: if it is missing, every op raises.
"""
from __future__ import annotations

import ctypes
import os
import re
import threading

import torch

_PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(_PKG_ROOT, "lib", "libwbk.so")
HEADER_PATH = os.path.join(os.path.dirname(_PKG_ROOT), "include", "wbk.h")

WBK_OK = 0
WBK_ERR_INVALID_ARG = 1
WBK_ERR_UNSUPPORTED = 2
WBK_ERR_CUDA = 3
WBK_ERR_DEVICE_TIMEOUT = 4

FMT_E4M3 = 0
FMT_E5M2 = 1

EPI_NONE = 0
EPI_GELU = 1
EPI_RESIDUAL = 2
EPI_RESIDUAL_CLAMP = 3
EPI_BIAS_MAXKEY = 4

_vp, _i64, _i32, _u64, _f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_uint64, ctypes.c_float

# name -> (restype, argtypes); mirrors include/wbk.h
_PROTOTYPES = {
    "wbk_version": (_i32, []),
    "wbk_last_error": (ctypes.c_char_p, []),
    "wbk_device_error": (_i32, [_vp]),
    "wbk_set_wait_timeout_ns": (_i32, [_u64]),
    "wbk_selftest_bounded_wait": (_i32, [_u64, _vp]),
    "wbk_amax_f16": (_i32, [_vp, _i64, _vp, _vp]),
    "wbk_quantise_from_amax_f16": (_i32, [_vp, _i64, _i32, _vp, _vp, _vp, _vp]),
    "wbk_quantise_f16": (_i32, [_vp, _i64, _i32, _vp, _vp, _vp, _vp]),
    "wbk_quantise_f16_noalloc": (_i32, [_vp, _i64, _i32, _vp, _vp, _vp]),
    "wbk_quantise_f16_resident": (_i32, [_vp, _i64, _i32, _vp, _vp, _vp, _vp, _vp]),
    "wbk_quantise_gelu_f16": (_i32, [_vp, _i64, _i32, _vp, _vp, _vp, _vp, _vp]),
    "wbk_scale_from_amax": (_i32, [_vp, _i32, _vp, _vp]),
    "wbk_layernorm_quantise_f16": (_i32, [_vp, _vp, _vp, _i64, _i64, _f32, _i32, _vp, _vp, _vp, _vp, _vp]),
    "wbk_layernorm_quantise_ws_bytes": (_i64, [_i64]),
    "wbk_dequantise_f16": (_i32, [_vp, _i64, _i32, _f32, _vp, _vp]),
    "wbk_layernorm_f16": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _f32, _vp, _vp]),
    "wbk_rmsnorm_f16": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _f32, _vp]),
    "wbk_gemm_fp8": (_i32, [_vp, _vp, _i64, _i64, _i64, _i32, _i32, _f32, _vp, _vp, _vp, _vp, _vp, _i32, _vp, _vp]),
    "wbk_attention_f16": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _f32, _vp, _vp]),
    "wbk_gemm_fp8_ws": (_i32, [_vp, _vp, _i64, _i64, _i64, _i32, _i32, _f32, _vp, _vp, _vp, _vp, _vp, _i32, _vp,
                               _vp, _i64, _vp]),
    "wbk_gemm_fp8_ws_bytes": (_i64, [_i64, _i64, _i64]),
    "wbk_linear_fp8_f16": (_i32, [_vp, _i64, _i64, _i64, _i32, _vp, _vp, _vp, _vp, _i32, _vp, _f32, _vp, _vp, _vp,
                                  _i32, _vp, _vp, _i64, _vp]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class WbkError(RuntimeError):
    """A libwbk call returned a non-zero status."""

    def __init__(self, what: str, status: int, message: str):
        super().__init__(f"{what}: {message} (wbk status {status})")
        self.status = status


def lib() -> ctypes.CDLL:
    """The loaded libwbk.so with typed prototypes (loaded once per process)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(
                        f"libwbk.so is not built ({LIB_PATH}); run `python whisper-blaze_b200/csrc/build.py`")
                L = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in _PROTOTYPES.items():
                    fn = getattr(L, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = L
    return _lib


def header_symbols() -> list[str]:
    """Names of every entry point declared in include/wbk.h."""
    with open(HEADER_PATH) as f:
        text = f.read()
    return sorted(set(re.findall(r"^\s*(?:const\s+char\s*\*|int64_t|int)\s+(wbk_\w+)\s*\(", text, flags=re.M)))


def check(status: int, what: str) -> None:
    if status != WBK_OK:
        msg = lib().wbk_last_error()
        raise WbkError(what, status, msg.decode() if msg else "")


def stream_of(t: torch.Tensor) -> int:
    """Raw cudaStream_t of torch's current stream on t's device."""
    return torch.cuda.current_stream(t.device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


_TIMEOUT_HOOKS: list = []


def on_device_timeout(fn):
    """Register fn(device_index), run by device_error() when it reports a device-side
    timeout on that device (e.g. to zero workspaces whose sync words a kernel that
    gave up left behind). Usable as a decorator."""
    _TIMEOUT_HOOKS.append(fn)
    return fn


def device_error() -> int:
    """Read and clear the device-side error word of the current device (syncs).

    The word is WBK_ERR_DEVICE_TIMEOUT | site << 8 after a bounded wait gave up.
    A kernel that gave up may leave the sync words and split-K tickets of its
    workspace non-zero, so on a timeout the registered hooks run first (the
    library's own shared workspaces are zeroed again by ops)."""
    code = ctypes.c_uint32(0)
    check(lib().wbk_device_error(ctypes.byref(code)), "wbk_device_error")
    if (code.value & 0xFF) == WBK_ERR_DEVICE_TIMEOUT:
        dev = torch.cuda.current_device()
        for fn in _TIMEOUT_HOOKS:
            fn(dev)
    return code.value


def set_wait_timeout_ns(timeout_ns: int) -> None:
    """Limit of every bounded device wait for later launches (0 = the default)."""
    check(lib().wbk_set_wait_timeout_ns(int(timeout_ns)), "wbk_set_wait_timeout_ns")
