"""CPU restatement of the FP8 linear (test infrastructure only).

The reference's FP8 linear (BlazeLinear.forward, whisper_blaze/model.py:80-109)
computes F.linear(dq(q8(x)), dq(q8(W)), bias); its unbound Hopper kernel
(csrc/kernels/gemm_hopper.cu:251-268) states the same product as
fp16(acc * (w_scale * a_scale) + bias). The oracle is that product with both
operands dequantised in fp32 (not rounded to fp16) and an fp32 torch-CPU
matmul, followed by the epilogue and one rounding to fp16:

  none      y = A W^T + bias
  gelu      y = gelu_erf(A W^T + bias)                 (HF activation "gelu")
  residual  y = A W^T + bias + residual
  clamp     y = clamp(A W^T + bias + residual, +-(65504 - 1000))
            (the fp16 clamp at the end of HF WhisperEncoderLayer.forward)
"""
from __future__ import annotations

import numpy as np
import torch

from . import fp8

EPI_NONE, EPI_GELU, EPI_RESIDUAL, EPI_RESIDUAL_CLAMP = 0, 1, 2, 3
EPILOGUES = {"none": EPI_NONE, "gelu": EPI_GELU, "residual": EPI_RESIDUAL, "residual_clamp": EPI_RESIDUAL_CLAMP}
FP16_CLAMP = 65504.0 - 1000.0


def dequant_tensor(q: torch.Tensor, scale: float, fmt: int = fp8.E4M3) -> torch.Tensor:
    """uint8 codes (CPU tensor) -> fp32 tensor of value * scale."""
    vals = torch.from_numpy(fp8._DECODE[fmt].copy())
    return vals[q.to(torch.int64)] * torch.tensor(np.float32(scale))


def gemm_fp8_ref_f32(a_q: torch.Tensor, a_scale: float, w_q: torch.Tensor, w_scale: float,
                     bias: torch.Tensor | None = None, residual: torch.Tensor | None = None,
                     epilogue: int = EPI_NONE, a_fmt: int = fp8.E4M3, w_fmt: int = fp8.E4M3) -> torch.Tensor:
    """fp32 result before the final fp16 rounding. a_q [M,K], w_q [N,K] uint8."""
    A = dequant_tensor(a_q.cpu(), a_scale, a_fmt)
    W = dequant_tensor(w_q.cpu(), w_scale, w_fmt)
    y = A @ W.t()
    if bias is not None:
        y = y + bias.cpu().float()
    if epilogue == EPI_GELU:
        y = torch.nn.functional.gelu(y)
    elif epilogue in (EPI_RESIDUAL, EPI_RESIDUAL_CLAMP):
        y = y + residual.cpu().float()
        if epilogue == EPI_RESIDUAL_CLAMP:
            y = y.clamp(-FP16_CLAMP, FP16_CLAMP)
    return y


def gemm_fp8_ref(*args, **kwargs) -> torch.Tensor:
    """fp16 result of gemm_fp8_ref_f32."""
    return gemm_fp8_ref_f32(*args, **kwargs).half()


def gelu_f16(y16: torch.Tensor) -> torch.Tensor:
    """fp16(gelu_erf(float(y))) for an fp16 tensor: HF's "gelu" on the fp16 fc1
    output, rounded to fp16 (the encoder's FFN activation)."""
    return torch.nn.functional.gelu(y16.float().cpu()).half()


def order_key_f16(v: float) -> int:
    """Order-preserving uint key of an fp16 value (the GEMM max-key epilogue's encoding)."""
    h = int(np.array([v], dtype=np.float16).view(np.uint16)[0])
    return (~h & 0xFFFF) if (h & 0x8000) else (h | 0x8000)


def rel_error(y: torch.Tensor, ref: torch.Tensor) -> float:
    """max|y - ref| / max|ref| over the whole output (the GEMM parity metric)."""
    y = y.float().cpu()
    ref = ref.float().cpu()
    denom = ref.abs().max().item()
    return (y - ref).abs().max().item() / (denom if denom > 0 else 1.0)
