"""C-ABI and host-logic checks that need no GPU.

libwbk.so must load and export every entry point include/wbk.h declares, and
its argument validation must reject bad calls before anything is launched
(those paths make no CUDA call, so they run here).
"""
import ctypes

import pytest
import torch

from whisper_blaze_b200 import _lib


def test_library_loads_and_exports_every_header_symbol():
    L = _lib.lib()
    names = _lib.header_symbols()
    assert len(names) >= 11
    for n in names:
        assert hasattr(L, n), f"libwbk.so does not export {n}"
    assert set(names) == set(_lib._PROTOTYPES), "ctypes prototypes out of sync with include/wbk.h"
    assert L.wbk_version() >= 10000


def _err(status):
    return status, _lib.lib().wbk_last_error().decode()


def test_gemm_rejects_bad_arguments_on_host():
    L = _lib.lib()
    fake = 0x10000  # never dereferenced: validation fails first
    st, msg = _err(L.wbk_gemm_fp8(fake, fake, 64, 64, 24, 0, 0, 1.0, None, None, None, None, fake, 0, None, None))
    assert st == _lib.WBK_ERR_UNSUPPORTED and "multiple of 16" in msg
    st, msg = _err(L.wbk_gemm_fp8(fake, fake, 64, 64, 32, 7, 0, 1.0, None, None, None, None, fake, 0, None, None))
    assert st == _lib.WBK_ERR_INVALID_ARG and "format" in msg
    st, msg = _err(L.wbk_gemm_fp8(fake, fake, 64, 64, 32, 0, 0, 1.0, None, None, None, None, fake, 2, None, None))
    assert st == _lib.WBK_ERR_INVALID_ARG and "residual" in msg
    st, msg = _err(L.wbk_gemm_fp8(fake, fake, 64, 64, 32, 0, 0, 1.0, None, None, None, None, fake, 9, None, None))
    assert st == _lib.WBK_ERR_INVALID_ARG and "epilogue" in msg
    st, msg = _err(L.wbk_gemm_fp8(fake + 1, fake, 64, 64, 32, 0, 0, 1.0, None, None, None, None, fake, 0, None, None))
    assert st == _lib.WBK_ERR_UNSUPPORTED and "aligned" in msg
    # M == 0 is a valid no-op
    assert L.wbk_gemm_fp8(None, None, 0, 64, 32, 0, 0, 1.0, None, None, None, None, None, 0, None, None) == 0


def test_quantiser_and_norm_reject_bad_arguments_on_host():
    L = _lib.lib()
    fake = 0x10000
    assert _err(L.wbk_quantise_f16(fake, 16, 5, fake, fake, fake, None))[0] == _lib.WBK_ERR_INVALID_ARG
    assert _err(L.wbk_quantise_f16(fake, -1, 0, fake, fake, fake, None))[0] == _lib.WBK_ERR_INVALID_ARG
    assert _err(L.wbk_quantise_f16(fake, 16, 0, fake, fake, None, None))[0] == _lib.WBK_ERR_INVALID_ARG
    assert _err(L.wbk_dequantise_f16(fake, 16, 3, 1.0, fake, None))[0] == _lib.WBK_ERR_INVALID_ARG
    st, msg = _err(L.wbk_layernorm_f16(fake, None, fake, fake, fake, None, 4, 100, 1e-5, None, None))
    assert st == _lib.WBK_ERR_UNSUPPORTED and "multiple of 8" in msg
    st, msg = _err(L.wbk_layernorm_f16(fake + 8, None, fake, fake, fake, None, 4, 128, 1e-5, None, None))
    assert st == _lib.WBK_ERR_UNSUPPORTED and "aligned" in msg
    assert _err(L.wbk_rmsnorm_f16(fake, None, fake, fake, 4, 128, 1e-5, None))[0] == _lib.WBK_ERR_INVALID_ARG
    assert _err(L.wbk_selftest_bounded_wait(0, None))[0] == _lib.WBK_ERR_INVALID_ARG
    # zero-size calls are valid no-ops
    assert L.wbk_dequantise_f16(None, 0, 0, 1.0, None, None) == 0
    assert L.wbk_amax_f16(None, 0, fake, None) == 0


def test_python_surface_checks_before_any_launch():
    import whisper_blaze_kernels as K
    x = torch.randn(16, 16).half()  # CPU tensor
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        K.quantise_e4m3(x)
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        K.layernorm_fused(x, None, torch.ones(16).half(), torch.zeros(16).half())
    x4 = torch.randn(1, 2, 16, 64).half()
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        K.encoder_self_attn(x4, x4, x4)
    with pytest.raises(NotImplementedError):
        K.decoder_self_attn(x4, x4, x4)
    with pytest.raises(NotImplementedError):
        K.mel_spectrogram(torch.zeros(16000))
    for name in ("quantise_e4m3", "quantise_e5m2", "dequantise_e4m3", "dequantise_e5m2", "layernorm_fused",
                 "layernorm_fused_residual", "rmsnorm_fused", "mel_spectrogram", "encoder_self_attn",
                 "decoder_cross_attn", "decoder_self_attn", "gemm_fp8_e4m3"):
        assert callable(getattr(K, name))


def test_layernorm_signature_matches_reference():
    import inspect
    import whisper_blaze_kernels as K
    params = list(inspect.signature(K.layernorm_fused).parameters)
    assert params == ["x", "residual", "gamma", "beta", "epsilon"]
    assert list(inspect.signature(K.rmsnorm_fused).parameters) == ["x", "residual", "gamma", "epsilon"]
    assert list(inspect.signature(K.dequantise_e4m3).parameters) == ["fp8", "scale", "shape"]
    assert list(inspect.signature(K.quantise_e4m3).parameters) == ["fp16"]
