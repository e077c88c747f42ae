"""Failure handling of the GEMM kernels on one GPU, without a fault or a hang.

Every mbarrier wait in the tcgen05 GEMM is bounded. A wait that runs out
records WBK_ERR_DEVICE_TIMEOUT | site << 8 in the device error word, raises the
CTA's abort flag so the other roles leave their loops, lets the loads and MMAs
already in flight land (bounded waits), frees TMEM and returns. These tests run
that path for real: wbk_set_wait_timeout_ns(1) makes the next launches give up
at their first wait that is not already complete, and the host reads the
status back. Nothing here faults, traps or spins without a limit; the drains
themselves are bounded at 1 ms.

Only the single-CTA kernel is driven into its abort path here (128-wide tiles:
1024 x 1024 x 4096 is one round of 64 tiles, which the host runs on single CTAs).
The CTA-pair kernel's abort path is not exercised on a GPU.

A kernel that gave up may leave the sync words and split-K tickets of its
workspace non-zero; device_error() then zeroes the library's shared workspaces
(ops._zero_shared_workspaces), which the second test checks with a forced
timeout from the bounded-wait self-test.
"""
import pytest
import torch

from conftest import randn_f16
from oracle import gemm
from whisper_blaze_b200 import _lib, ops

pytestmark = pytest.mark.gpu

GEMM_SITES = range(1, 8)  # SITE_PRODUCER_EMPTY .. SITE_EPI_RES of wbk_gemm.cu


def _operands(M, N, K, seed, dev):
    aq, sa = ops.quantise(randn_f16((M, K), seed).to(dev))
    wq, sw = ops.quantise(randn_f16((N, K), seed + 1, std=0.02).to(dev))
    b = randn_f16((N,), seed + 2, std=0.02).to(dev)
    return aq, sa, wq, sw, b


def _oracle(aq, sa, wq, sw, b):
    return gemm.gemm_fp8_ref_f32(aq.cpu(), float(sa.item()), wq.cpu(), float(sw.item()), b.cpu())


def test_gemm_gives_up_with_a_status_and_the_next_gemm_is_correct(cuda_device):
    M, N, K = 1024, 1024, 4096
    aq, sa, wq, sw, b = _operands(M, N, K, 3, cuda_device)
    assert _lib.device_error() == 0
    code = 0
    try:
        _lib.set_wait_timeout_ns(1)
        # A 1 ns limit makes the first wait that is not complete at once give up; which
        # wait that is depends on timing, so allow a few launches for one to happen.
        for _ in range(10):
            ops.gemm_fp8(aq, sa, wq, sw, b)
            code = _lib.device_error()
            if code:
                break
    finally:
        _lib.set_wait_timeout_ns(0)
    assert code & 0xFF == _lib.WBK_ERR_DEVICE_TIMEOUT, f"no device timeout reported (word {code:#x})"
    assert (code >> 8) in GEMM_SITES, f"site {code >> 8} is not a GEMM wait site"
    # the context is intact and the kernel, with the default limit, is exact again
    y = ops.gemm_fp8(aq, sa, wq, sw, b)
    assert _lib.device_error() == 0
    ref = _oracle(aq, sa, wq, sw, b)
    assert gemm.rel_error(y, ref) <= 1e-2
    assert torch.equal(y, ops.gemm_fp8(aq, sa, wq, sw, b))


def test_timeout_zeroes_the_shared_workspace_for_the_next_linear(cuda_device):
    """A stale arrival count in the shared workspace would let the next one-call linear pass
    its grid-wide arrivals early and quantise with a partial amax, silently. After
    device_error() reports a timeout, the workspace is zero again and the linear exact."""
    M, N, K = 64, 1280, 1280
    x = randn_f16((M, K), 40).to(cuda_device)
    wq, sw = ops.quantise(randn_f16((N, K), 41, std=0.02).to(cuda_device))
    b = randn_f16((N,), 42, std=0.02).to(cuda_device)
    y0, q0, s0 = ops.linear_fp8(x, wq, sw, b)  # creates the device's shared workspace
    ws = ops._SPLITK_WS[cuda_device]
    ws[:64].fill_(0x5A)  # what a linear that gave up between its arrivals could leave behind
    _lib.check(_lib.lib().wbk_selftest_bounded_wait(20_000_000, _lib.stream_of(x)), "selftest")
    code = _lib.device_error()
    assert code & 0xFF == _lib.WBK_ERR_DEVICE_TIMEOUT
    assert int(ws.count_nonzero().item()) == 0
    y1, q1, s1 = ops.linear_fp8(x, wq, sw, b)
    assert torch.equal(q1, q0) and torch.equal(s1, s0)
    assert torch.equal(y1.view(torch.int16), y0.view(torch.int16))
    ref = gemm.gemm_fp8_ref_f32(q1.cpu(), float(s1.item()), wq.cpu(), float(sw.item()), b.cpu())
    assert gemm.rel_error(y1, ref) <= 1e-2
    assert _lib.device_error() == 0
