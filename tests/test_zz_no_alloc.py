"""wbk_quantise_f16_noalloc: the quantise entry point for callers that cannot allocate.

Some callers of this library run where they may not call cudaMalloc (a host
callback or real-time audio thread with a no-allocation rule, a plugin whose
host owns every device allocation). The no-allocation entry point keeps its
scratch in a static device array instead of a caller-provided buffer; these
tests call it through the C ABI and check it against wbk_quantise_f16 — the
fp8 bytes and the scale bit for bit, the tolerance every quantiser test here
uses — on two calls in a row (the second must not see the first's scratch),
and check that a tensor beyond the static scratch's limit is refused before
any launch. This file is named to be collected last.
"""
import pytest
import torch

from conftest import randn_f16
from whisper_blaze_b200 import _lib

pytestmark = pytest.mark.gpu

NOALLOC_MAX_ELEMS = 65536 * 4095


def _quantise_reference(x, fmt):
    q = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    s = torch.empty(1, dtype=torch.float32, device=x.device)
    ws = torch.empty(1, dtype=torch.int32, device=x.device)
    _lib.check(_lib.lib().wbk_quantise_f16(x.data_ptr(), x.numel(), fmt, q.data_ptr(), s.data_ptr(), ws.data_ptr(),
                                           _lib.stream_of(x)), "wbk_quantise_f16")
    return q, s


def _quantise_noalloc(x, fmt):
    q = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    s = torch.empty(1, dtype=torch.float32, device=x.device)
    _lib.check(_lib.lib().wbk_quantise_f16_noalloc(x.data_ptr(), x.numel(), fmt, q.data_ptr(), s.data_ptr(),
                                                   _lib.stream_of(x)), "wbk_quantise_f16_noalloc")
    return q, s


@pytest.mark.parametrize("fmt", [_lib.FMT_E4M3, _lib.FMT_E5M2])
def test_noalloc_matches_existing_entry_point_on_consecutive_calls(cuda_device, fmt):
    # a large-amax tensor spanning many CTAs, then a small-amax ragged one: the
    # second call must not inherit anything from the first call's scratch
    first = randn_f16((1500, 1280), 500) * 8
    second = randn_f16((4099,), 501, std=0.01)
    # then a view one element into its buffer (not 16-byte aligned: the element-wise
    # partial-max kernel and quantise path) spanning several CTAs, and an empty tensor
    # (one CTA over an empty range: amax 0, scale 1)
    shifted = randn_f16((200001,), 502, std=3.0).to(cuda_device)[1:]
    assert shifted.data_ptr() % 16 != 0
    empty = torch.empty(0, dtype=torch.float16, device=cuda_device)
    for x in (first.to(cuda_device), second.to(cuda_device), shifted, empty):
        q_ref, s_ref = _quantise_reference(x, fmt)
        q, s = _quantise_noalloc(x, fmt)
        torch.cuda.synchronize()
        assert torch.equal(q, q_ref), "fp8 bytes differ from wbk_quantise_f16"
        assert s.view(torch.int32).item() == s_ref.view(torch.int32).item(), "scale differs from wbk_quantise_f16"
    assert _lib.device_error() == 0


def test_noalloc_rejects_tensors_beyond_its_static_scratch(cuda_device):
    x = torch.zeros(16, dtype=torch.float16, device=cuda_device)
    q = torch.empty(16, dtype=torch.uint8, device=cuda_device)
    s = torch.empty(1, dtype=torch.float32, device=cuda_device)
    L = _lib.lib()
    # the size check runs on the host before any launch, so a short buffer is never touched
    st = L.wbk_quantise_f16_noalloc(x.data_ptr(), NOALLOC_MAX_ELEMS + 1, _lib.FMT_E4M3, q.data_ptr(), s.data_ptr(),
                                    _lib.stream_of(x))
    assert st == _lib.WBK_ERR_UNSUPPORTED
    assert b"exceeds the limit" in L.wbk_last_error()
