"""GPU parity of the one-call FP8 linear (wbk_linear_fp8_f16 through ops.linear_fp8).

For M <= 128 the GEMM quantises its fp16 activation itself (cooperative
launch: grid-wide amax, then codes), replacing the quantise + GEMM pair that
BlazeLinear.forward issues per FP8 linear (whisper_blaze/model.py:80-109).
Gates: the codes, scale and amax bits equal the standalone quantiser's bit for
bit (and the reference's golden vectors); the output equals gemm_fp8 on those
codes bit for bit, for every epilogue and both formats; the output is within
the north-star max relative error 1e-2 of the fp32 oracle; the workspace's
sync words are zero again after every call.
"""
import os

import numpy as np
import pytest
import torch

from conftest import randn_f16
from oracle import fp8, gemm
from whisper_blaze_b200 import _lib, ops

pytestmark = pytest.mark.gpu

GOLDEN_DIR = os.path.join(os.path.dirname(__file__), "golden")


def _bits(t: torch.Tensor) -> int:
    return int(np.float32(t.item()).view(np.int32))


def _check_linear(x, wq, sw, b=None, res=None, epilogue="none", a_fmt="e4m3", w_fmt="e4m3", ws=None):
    dev = x.device
    key_f = ops.new_amax_ws(dev) if epilogue == "bias_maxkey" else None
    key_u = ops.new_amax_ws(dev) if epilogue == "bias_maxkey" else None
    out_f = torch.full(x.shape[:-1] + (wq.shape[0],), float("nan"), dtype=torch.float16, device=dev)
    amax_f = torch.full((1,), -1, dtype=torch.int32, device=dev)
    y, q, s = ops.linear_fp8(x, wq, sw, b, res, epilogue, a_format=a_fmt, w_format=w_fmt, out=out_f,
                             out_amax=key_f, amax_ws=amax_f, workspace=ws)
    q_ref, s_ref = ops.quantise(x, a_fmt)
    assert torch.equal(q, q_ref), "codes differ from the standalone quantiser"
    assert _bits(s) == _bits(s_ref), (s.item(), s_ref.item())
    finite_abs = x.float().abs().nan_to_num(nan=0.0, posinf=float("inf"))
    amax_ref = finite_abs.max().half().view(torch.int16).item() & 0xFFFF
    assert (int(amax_f.item()) & 0xFFFF) == amax_ref
    y_ref = ops.gemm_fp8(q_ref, s_ref, wq, sw, b, res, epilogue, a_format=a_fmt, w_format=w_fmt, out_amax=key_u)
    assert torch.equal(y.view(torch.int16), y_ref.view(torch.int16)), "output differs from gemm_fp8 on the same codes"
    if key_f is not None:
        assert key_f.item() == key_u.item()
    return y, q, s


def _weights(N, K, seed, dev, fmt="e4m3"):
    w = randn_f16((N, K), seed, std=0.02).to(dev)
    return ops.quantise(w, fmt)


@pytest.mark.parametrize("M,N,K", [(1, 1280, 1280), (8, 24, 64), (17, 640, 1296), (64, 1280, 1280),
                                   (64, 3840, 1280), (64, 5120, 1280), (100, 1000, 512), (128, 2560, 1280),
                                   (16, 1280, 5120), (32, 1280, 5120), (64, 1280, 5120)])
def test_linear_matches_quantise_then_gemm(cuda_device, M, N, K):
    x = randn_f16((M, K), M + N + K).to(cuda_device)
    wq, sw = _weights(N, K, 7, cuda_device)
    b = randn_f16((N,), 8, std=0.02).to(cuda_device)
    y, q, s = _check_linear(x, wq, sw, b)
    ref = gemm.gemm_fp8_ref_f32(q.cpu(), float(s.item()), wq.cpu(), float(sw.item()), b.cpu(), None, gemm.EPI_NONE,
                                fp8.E4M3, fp8.E4M3)
    err = ((y.float().cpu() - ref).abs().max() / ref.abs().max()).item()
    assert err <= 1e-2, f"max relative error {err:.3e}"


def test_linear_vocab_projection(cuda_device):
    """The decoder step's logits projection: N = 51866 (ragged last tile), 811 tiles on 148 CTAs."""
    x = randn_f16((64, 1280), 3).to(cuda_device)
    wq, sw = _weights(51866, 1280, 4, cuda_device)
    _check_linear(x, wq, sw)


@pytest.mark.parametrize("epilogue", ["none", "gelu", "residual", "residual_clamp", "bias_maxkey"])
@pytest.mark.parametrize("M,N,K", [(64, 1280, 1280), (5, 200, 256)])
def test_linear_epilogues(cuda_device, epilogue, M, N, K):
    x = randn_f16((M, K), 11).to(cuda_device)
    wq, sw = _weights(N, K, 12, cuda_device)
    b = randn_f16((N,), 13, std=0.02).to(cuda_device)
    res = randn_f16((M, N), 14).to(cuda_device) if epilogue.startswith("residual") else None
    _check_linear(x, wq, sw, b, res, epilogue)


@pytest.mark.parametrize("a_fmt,w_fmt", [("e5m2", "e4m3"), ("e4m3", "e5m2"), ("e5m2", "e5m2")])
def test_linear_formats(cuda_device, a_fmt, w_fmt):
    x = randn_f16((48, 1024), 21, std=30.0).to(cuda_device)
    wq, sw = _weights(768, 1024, 22, cuda_device, w_fmt)
    _check_linear(x, wq, sw, a_fmt=a_fmt, w_fmt=w_fmt)


def test_linear_special_values(cuda_device):
    """Zeros (scale 1), NaN (ignored by the amax, coded -max), +-inf and the fp16 extremes."""
    wq, sw = _weights(256, 512, 31, cuda_device)
    zeros = torch.zeros(16, 512, dtype=torch.float16, device=cuda_device)
    _, _, s = _check_linear(zeros, wq, sw)
    assert s.item() == 1.0
    x = randn_f16((16, 512), 32).to(cuda_device)
    x[0, 0] = float("nan")
    x[1, 5] = 65504.0
    x[2, 7] = -65504.0
    x[3, 9] = 6e-8
    _check_linear(x, wq, sw)


def test_linear_golden_codes(cuda_device):
    """The reference quantiser's golden bytes and scales, produced by the in-kernel quantise."""
    path = os.path.join(GOLDEN_DIR, "ref_quantise.npz")
    g = np.load(path)
    for name in sorted({k.split("__")[0] for k in g.files}):
        x = torch.from_numpy(g[f"{name}__x"])
        x2 = x if x.dim() == 2 else x.reshape(-1, 128)
        if x2.shape[0] > 128 or x2.shape[1] % 16:
            continue
        wq, sw = _weights(64, x2.shape[1], 41, cuda_device)
        for fmt_name in ("e4m3", "e5m2"):
            _, q, s = ops.linear_fp8(x2.contiguous().to(cuda_device), wq, sw, a_format=fmt_name)
            assert np.array_equal(q.cpu().numpy().reshape(-1), g[f"{name}__q_{fmt_name}"].reshape(-1)), \
                f"{name} {fmt_name} bytes"
            assert _bits(s) == int(np.float32(g[f"{name}__s_{fmt_name}"]).view(np.int32))


def test_linear_workspace_reusable_and_deterministic(cuda_device):
    """One workspace across shapes and calls: sync words back at zero, repeated calls bit-identical."""
    ws = torch.zeros(8 << 20, dtype=torch.uint8, device=cuda_device)
    shapes = [(64, 1280, 1280), (16, 1280, 5120), (3, 520, 96), (64, 51866, 1280), (128, 640, 640)]
    first = {}
    for rep in range(2):
        for (M, N, K) in shapes:
            x = randn_f16((M, K), M * 7 + K).to(cuda_device)
            wq, sw = _weights(N, K, N % 97, cuda_device)
            y, q, s = ops.linear_fp8(x, wq, sw, workspace=ws)
            torch.cuda.synchronize()
            assert int(ws[:256].view(torch.int32).abs().sum().item()) == 0, "sync words not reset"
            if rep == 0:
                first[(M, N, K)] = (y.clone(), q.clone(), s.clone())
            else:
                y0, q0, s0 = first[(M, N, K)]
                assert torch.equal(y.view(torch.int16), y0.view(torch.int16))
                assert torch.equal(q, q0) and _bits(s) == _bits(s0)
    assert _lib.device_error() == 0


def test_linear_large_m_uses_two_launches(cuda_device):
    """M > 128: the quantiser kernel then the GEMM, same contract."""
    x = randn_f16((300, 512), 51).to(cuda_device)
    wq, sw = _weights(384, 512, 52, cuda_device)
    _check_linear(x, wq, sw)


def test_linear_in_cuda_graph(cuda_device):
    """Captured once, replayed: the cooperative launch works inside a graph and resets its words."""
    x = randn_f16((64, 1280), 61).to(cuda_device)
    wq, sw = _weights(3840, 1280, 62, cuda_device)
    ws = torch.zeros(4096, dtype=torch.uint8, device=cuda_device)
    out = torch.empty(64, 3840, dtype=torch.float16, device=cuda_device)
    q = torch.empty(64, 1280, dtype=torch.uint8, device=cuda_device)
    s = torch.empty(1, dtype=torch.float32, device=cuda_device)
    a = torch.empty(1, dtype=torch.int32, device=cuda_device)
    st = torch.cuda.Stream(cuda_device)
    with torch.cuda.stream(st):
        ops.linear_fp8(x, wq, sw, out=out, q_out=q, scale_out=s, amax_ws=a, workspace=ws)  # warm-up, outside capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        ops.linear_fp8(x, wq, sw, out=out, q_out=q, scale_out=s, amax_ws=a, workspace=ws)
    for seed in (63, 64, 65):
        x.copy_(randn_f16((64, 1280), seed).to(cuda_device))
        g.replay()
        torch.cuda.synchronize()
        q_ref, s_ref = ops.quantise(x)
        y_ref = ops.gemm_fp8(q_ref, s_ref, wq, sw)
        assert torch.equal(q, q_ref) and _bits(s) == _bits(s_ref)
        assert torch.equal(out.view(torch.int16), y_ref.view(torch.int16))
        assert int(ws[:256].view(torch.int32).abs().sum().item()) == 0
    del g


def test_linear_argument_errors(cuda_device):
    x = randn_f16((4, 64), 1).to(cuda_device)
    wq, sw = _weights(32, 64, 2, cuda_device)
    with pytest.raises(RuntimeError, match="K="):
        ops.linear_fp8(randn_f16((4, 48), 1).to(cuda_device), wq, sw)
    with pytest.raises(RuntimeError, match="residual"):
        ops.linear_fp8(x, wq, sw, epilogue="residual")
    with pytest.raises(RuntimeError, match="workspace"):
        ops.linear_fp8(x, wq, sw, workspace=torch.zeros(64, dtype=torch.uint8, device=cuda_device))
