"""CPU checks of the norm and GEMM oracles (no GPU).

The LayerNorm / RMSNorm oracles are pinned by the reference's own norm tests
(tests/test_kernels.py:86-150, :191-213 of whisper-blaze), restated here, and
by golden outputs of the reference's CUDA norm kernels (tests/golden/).
"""
import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from conftest import GOLDEN_DIR, randn_f16
from oracle import fp8, gemm, norm

ATOL, RTOL = 1e-2, 1e-1  # the reference test tolerances (tests/test_kernels.py:34-35)


def test_ref_layernorm_matches_torch():
    x, res = randn_f16((128, 1280), 10), randn_f16((128, 1280), 11)
    g, b = torch.ones(1280, dtype=torch.float16), torch.zeros(1280, dtype=torch.float16)
    out = norm.layernorm_ref(x, res, g, b).half().float()
    ref = F.layer_norm((x + res).float(), [1280], g.float(), b.float(), 1e-5)
    assert torch.allclose(out, ref, atol=ATOL, rtol=RTOL)


def test_ref_layernorm_gamma_scaling():
    x = randn_f16((16, 512), 12)
    res = torch.zeros(16, 512, dtype=torch.float16)
    g, b = torch.full((512,), 2.0, dtype=torch.float16), torch.zeros(512, dtype=torch.float16)
    out = norm.layernorm_ref(x, res, g, b).half().float()
    assert torch.allclose(out, F.layer_norm(x.float(), [512], g.float(), b.float(), 1e-5), atol=ATOL, rtol=RTOL)


def test_ref_residual_sum_is_exact():
    x, res = randn_f16((128, 1280), 13), randn_f16((128, 1280), 14)
    assert torch.equal(norm.layernorm_sum_ref(x, res), x + res)


def test_ref_rmsnorm_formula():
    x, res = randn_f16((32, 512), 15), randn_f16((32, 512), 16)
    g = torch.ones(512, dtype=torch.float16)
    h = (x + res).float()  # the reference test adds in fp16 first
    ref = h * h.pow(2).mean(-1, keepdim=True).add(1e-5).rsqrt() * g.float()
    assert torch.allclose(norm.rmsnorm_ref(x, res, g).half().float(), ref, atol=ATOL, rtol=RTOL)


def test_ln_tolerance_shape():
    ref = torch.tensor([0.0, 0.5, 1.9, 2.0, 7.5, -6.0])
    tol = norm.ln_tolerance(ref)
    assert tol[0] == 1e-3 and tol[1] == 1e-3 and tol[2] == 1e-3
    assert tol[3] == 2.0 ** -9 and tol[4] == 2.0 ** -8 and tol[5] == 2.0 ** -8


GOLDEN_NORM = os.path.join(GOLDEN_DIR, "ref_norm.npz")


def test_golden_layernorm_vs_oracle():
    """The reference CUDA LayerNorm agrees with the oracle within the gate, and
    its sum output equals fp16(x + res) exactly."""
    if not os.path.exists(GOLDEN_NORM):
        pytest.fail(f"golden fixture {GOLDEN_NORM} is missing (tests/golden/make_golden.py on a B200)")
    g = np.load(GOLDEN_NORM)
    x, res, gam, bet = (torch.from_numpy(g[k]) for k in ("x", "res", "gamma", "beta"))
    ref = norm.layernorm_ref(x, res, gam, bet)
    out = torch.from_numpy(g["ln_out"]).float()
    assert ((out - ref).abs() <= norm.ln_tolerance(ref)).all()
    assert torch.equal(torch.from_numpy(g["ln_sum"]), norm.layernorm_sum_ref(x, res))
    rms_ref = norm.rmsnorm_ref(x, res, gam)
    rms = torch.from_numpy(g["rms_out"]).float()
    assert ((rms - rms_ref).abs() <= norm.ln_tolerance(rms_ref)).all()


# ---- GEMM oracle sanity

def test_gemm_oracle_identity_weight():
    K = 64
    x = randn_f16((8, K), 20)
    qa, sa = fp8.quantise(x.numpy(), fp8.E4M3)
    eye_q = fp8.encode_rne_satfinite(np.eye(K, dtype=np.float32), fp8.E4M3)
    y = gemm.gemm_fp8_ref(torch.from_numpy(qa), sa, torch.from_numpy(eye_q), 1.0)
    expect = torch.from_numpy(fp8.dequantise_f32(qa, sa, fp8.E4M3)).half()
    assert torch.equal(y, expect)


def test_gemm_oracle_epilogues():
    M, N, K = 16, 24, 32
    qa = torch.randint(0, 0x7E, (M, K), dtype=torch.uint8)
    qw = torch.randint(0, 0x7E, (N, K), dtype=torch.uint8)
    bias = randn_f16((N,), 21)
    res = randn_f16((M, N), 22)
    base = gemm.gemm_fp8_ref_f32(qa, 0.01, qw, 0.02, bias)
    assert torch.allclose(gemm.gemm_fp8_ref_f32(qa, 0.01, qw, 0.02, bias, epilogue=gemm.EPI_GELU), F.gelu(base))
    assert torch.allclose(gemm.gemm_fp8_ref_f32(qa, 0.01, qw, 0.02, bias, res, gemm.EPI_RESIDUAL),
                          base + res.float())


def test_rel_error_metric():
    ref = torch.tensor([1.0, -2.0, 4.0])
    assert gemm.rel_error(ref + torch.tensor([0.0, 0.04, 0.0]), ref) == pytest.approx(0.01)
