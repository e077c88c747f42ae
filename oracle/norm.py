"""CPU restatement of the fused residual + LayerNorm / RMSNorm (test infrastructure only).

Follows csrc/kernels/layernorm_fused.cu of whisper-blaze v0.1.17:
  layernorm_fused_kernel (:50-184): s = float(x) (+ float(res)); mean, then the
  variance of (s - mean), both over D in fp32; out = (s - mean) * rsqrt(var +
  eps) * gamma + beta; the optional second output is fp16(s).
  rmsnorm_fused_kernel (:191-258): out = (x + res) * rsqrt(mean((x+res)^2) + eps)
  * gamma, residual required.
The reference's own tests compare against F.layer_norm on (x + res) in fp32
(tests/test_kernels.py:96-103) and against that explicit RMS formula
(tests/test_kernels.py:208-213); these functions are exactly those
expressions, returned in fp32 (callers round to fp16 where they compare
stored outputs).
"""
from __future__ import annotations

import torch


def residual_sum(x: torch.Tensor, residual: torch.Tensor | None) -> torch.Tensor:
    s = x.float().cpu()
    if residual is not None:
        s = s + residual.float().cpu()
    return s


def layernorm_ref(x: torch.Tensor, residual: torch.Tensor | None, gamma: torch.Tensor, beta: torch.Tensor,
                  eps: float = 1e-5) -> torch.Tensor:
    s = residual_sum(x, residual)
    return torch.nn.functional.layer_norm(s, [s.shape[-1]], gamma.float().cpu(), beta.float().cpu(), eps)


def layernorm_sum_ref(x: torch.Tensor, residual: torch.Tensor | None) -> torch.Tensor:
    """The second output of layernorm_fused_residual: fp16(x + residual)."""
    return residual_sum(x, residual).half()


def rmsnorm_ref(x: torch.Tensor, residual: torch.Tensor, gamma: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    h = residual_sum(x, residual)
    rms = h.pow(2).mean(-1, keepdim=True).add(eps).rsqrt()
    return h * rms * gamma.float().cpu()


def fp16_ulp(v: torch.Tensor) -> torch.Tensor:
    """Spacing of the fp16 grid at |v| (normal range): 2^(floor(log2|v|) - 10)."""
    _, e = torch.frexp(v.float().abs())
    return torch.pow(2.0, (e - 11).float())


def ln_tolerance(ref: torch.Tensor) -> torch.Tensor:
    """Per-element LayerNorm gate: 1e-3 absolute, widened to one fp16 ulp of
    the reference value where the fp16 output grid itself is coarser than
    1e-3 (|ref| >= 2, where a correctly rounded fp16 output can already be
    ~1e-3 away): max(1e-3, ulp16(ref))."""
    return torch.clamp(fp16_ulp(ref), min=1e-3)
