"""Bounded device waits: a wait that runs out returns a status, the context stays usable.

The self-test kernel waits on an mbarrier that nothing ever arrives on, with a
short limit; the wait gives up, records WBK_ERR_DEVICE_TIMEOUT in the device
error word and the kernel returns. No fault, trap or hang is involved.
"""
import pytest
import torch

from whisper_blaze_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_with_status(cuda_device):
    assert _lib.device_error() == 0
    with torch.cuda.device(cuda_device):
        _lib.check(_lib.lib().wbk_selftest_bounded_wait(20_000_000, _lib.stream_of(torch.empty(1, device=cuda_device))),
                   "selftest")
        code = _lib.device_error()
    assert code & 0xFF == _lib.WBK_ERR_DEVICE_TIMEOUT
    assert (code >> 8) == 15  # the self-test site
    assert _lib.device_error() == 0  # reading cleared it
    # the context is still healthy: a GEMM runs and is correct afterwards
    from oracle import gemm
    g = torch.Generator().manual_seed(0)
    a = torch.randint(0, 0x30, (128, 256), dtype=torch.uint8, generator=g)  # |values| <= 0.5
    w = torch.randint(0, 0x30, (256, 256), dtype=torch.uint8, generator=g)
    y = ops.gemm_fp8(a.to(cuda_device), 1.0, w.to(cuda_device), 1.0)
    ref = gemm.gemm_fp8_ref_f32(a, 1.0, w, 1.0)
    assert gemm.rel_error(y, ref) <= 1e-2
