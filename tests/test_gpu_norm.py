"""GPU parity of LayerNorm / RMSNorm (calls go through the C ABI).

Gate: LayerNorm output within 1e-3 absolute of the fp32 oracle (widened to one
fp16 ulp where |ref| >= 2, see oracle.norm.ln_tolerance); the residual-sum
output bit-exact to fp16(x + residual).
"""
import pytest
import torch
import torch.nn.functional as F

from conftest import randn_f16
from oracle import norm
from whisper_blaze_b200 import ops

pytestmark = pytest.mark.gpu


def _params(D, seed):
    g = (1.0 + randn_f16((D,), seed, std=0.1).float()).half()
    b = randn_f16((D,), seed + 1, std=0.1)
    return g, b


def _check_ln(out, ref):
    err = (out.float().cpu() - ref).abs()
    tol = norm.ln_tolerance(ref)
    assert (err <= tol).all(), f"max err {err.max().item():.3e}, worst excess {(err - tol).max().item():.3e}"


@pytest.mark.parametrize("rows,D", [(1, 8), (7, 64), (128, 512), (1500, 1280), (33, 1288), (64, 4096),
                                    (5, 8192), (3, 20000)])
@pytest.mark.parametrize("with_res", [False, True])
def test_layernorm_matches_oracle(cuda_device, rows, D, with_res):
    x = randn_f16((rows, D), rows * 7 + D)
    res = randn_f16((rows, D), rows * 7 + D + 1) if with_res else None
    g, b = _params(D, D)
    dev = lambda t: None if t is None else t.to(cuda_device)  # noqa: E731
    out, s = ops.layernorm(dev(x), dev(res), dev(g), dev(b), 1e-5, want_sum=True)
    _check_ln(out, norm.layernorm_ref(x, res, g, b))
    assert torch.equal(s.cpu(), norm.layernorm_sum_ref(x, res))


def test_layernorm_amax_output(cuda_device):
    x = randn_f16((300, 1280), 5).to(cuda_device)
    g, b = (t.to(cuda_device) for t in _params(1280, 3))
    amax = ops.new_amax_ws(cuda_device)
    out, _ = ops.layernorm(x, None, g, b, out_amax=amax)
    expect = out.float().abs().max().half().view(torch.int16).item()
    assert amax.item() == expect


@pytest.mark.parametrize("rows,D", [(32, 512), (1500, 1280), (4, 8192)])
def test_rmsnorm_matches_oracle(cuda_device, rows, D):
    x, res = randn_f16((rows, D), 40), randn_f16((rows, D), 41)
    g = _params(D, 42)[0]
    out = ops.rmsnorm(x.to(cuda_device), res.to(cuda_device), g.to(cuda_device))
    _check_ln(out, norm.rmsnorm_ref(x, res, g))


# ---- the reference's own norm tests (tests/test_kernels.py:86-213) on the B200 kernels

def test_ref_suite_layernorm(cuda_device):
    import whisper_blaze_kernels as K
    ATOL, RTOL = 1e-2, 1e-1
    D = 1280
    x = torch.randn(128, D, dtype=torch.float16, device=cuda_device)
    res = torch.randn(128, D, dtype=torch.float16, device=cuda_device)
    g = torch.ones(D, dtype=torch.float16, device=cuda_device)
    b = torch.zeros(D, dtype=torch.float16, device=cuda_device)
    out = K.layernorm_fused(x, res, g, b, 1e-5)
    assert out.shape == x.shape
    assert torch.allclose(out.float(), F.layer_norm((x + res).float(), [D], g.float(), b.float(), 1e-5),
                          atol=ATOL, rtol=RTOL)
    out = K.layernorm_fused(x, None, g, b, 1e-5).float()
    assert torch.allclose(out, F.layer_norm(x.float(), [D], g.float(), b.float(), 1e-5), atol=ATOL, rtol=RTOL)
    x3 = torch.randn(2, 64, D, dtype=torch.float16, device=cuda_device)
    out3 = K.layernorm_fused(x3, None, g, b, 1e-5)
    assert out3.shape == x3.shape
    normed, total = K.layernorm_fused_residual(x, res, g, b, 1e-5)
    assert torch.equal(total, x + res)
    r = K.rmsnorm_fused(x[:, :512].contiguous(), res[:, :512].contiguous(), g[:512].contiguous(), 1e-5).float()
    h = (x[:, :512] + res[:, :512]).float()
    assert torch.allclose(r, h * h.pow(2).mean(-1, keepdim=True).add(1e-5).rsqrt(), atol=ATOL, rtol=RTOL)


def test_blaze_layernorm_module(cuda_device):
    from whisper_blaze_b200.modules import BlazeLayerNorm
    ln = torch.nn.LayerNorm(1280, eps=1e-5).to(cuda_device).half()
    torch.nn.init.normal_(ln.weight, mean=1.0, std=0.1)
    torch.nn.init.normal_(ln.bias, mean=0.0, std=0.1)
    blaze = BlazeLayerNorm.from_layernorm(ln)
    x = torch.randn(2, 64, 1280, dtype=torch.float16, device=cuda_device)
    assert torch.allclose(blaze(x).float(), ln(x).float(), atol=1e-2, rtol=1e-1)
    assert blaze(torch.randn(4, 1280, device=cuda_device)).dtype == torch.float32
    assert BlazeLayerNorm.supports(torch.nn.LayerNorm(1280))
    assert not BlazeLayerNorm.supports(torch.nn.LayerNorm(100))


def test_layernorm_matches_live_reference_kernel(cuda_device):
    """The reference's own CUDA LayerNorm / RMSNorm (oracle/_ref) on the same inputs."""
    from oracle import build_ref
    try:
        R = build_ref.load()
    except ImportError as e:
        pytest.skip(str(e))
    x, res = randn_f16((1500, 1280), 60).to(cuda_device), randn_f16((1500, 1280), 61).to(cuda_device)
    g, b = (t.to(cuda_device) for t in _params(1280, 62))
    ref_out, ref_sum = R.layernorm_fused_residual(x, res, g, b, 1e-5)
    out, s = ops.layernorm(x, res, g, b, 1e-5, want_sum=True)
    assert torch.equal(s, ref_sum)
    d = (out.float() - ref_out.float()).abs()
    assert (d <= norm.ln_tolerance(ref_out.float().cpu()).to(cuda_device)).all()
    r_ref = R.rmsnorm_fused(x, res, g, 1e-5)
    r = ops.rmsnorm(x, res, g, 1e-5)
    assert ((r.float() - r_ref.float()).abs() <= norm.ln_tolerance(r_ref.float().cpu()).to(cuda_device)).all()


@pytest.mark.parametrize("rows,D", [(1, 8), (7, 64), (1500, 1280), (333, 1288), (64, 4096),
                                    # many rows per warp: the row ring of both passes wraps several times
                                    (20000, 1280), (5003, 2056), (3001, 4096)])
@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_layernorm_quantise_is_bit_identical_to_unfused(cuda_device, rows, D, fmt):
    """The fused LayerNorm->FP8 path writes exactly the codes and scale of LayerNorm then quantise."""
    x = randn_f16((rows, D), 70 + rows).to(cuda_device) * 3
    g, b = (t.to(cuda_device) for t in _params(D, 71))
    ln, _ = ops.layernorm(x, None, g, b)
    q_ref, s_ref = ops.quantise(ln, fmt)
    q, s = ops.layernorm_quantise(x, g, b, fmt=fmt)
    assert s.view(torch.int32).item() == s_ref.view(torch.int32).item()
    assert torch.equal(q, q_ref)
