"""nn.Module equivalents of the reference's BlazeLinear and BlazeLayerNorm.

BlazeLinear mirrors whisper_blaze/model.py:47-109 (same constructor, buffers
and FP16 path) but its FP8 branch runs the B200 FP8 GEMM on the quantised
operands instead of dequantising both and calling an fp16 F.linear; the
weight is quantised once at construction and its scale stays on the device.
BlazeLayerNorm mirrors model.py:116-168 unchanged in behaviour.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from . import ops
from .precision import LayerPrecision


class BlazeLinear(nn.Module):
    """Linear layer whose FP8 precision runs on the tcgen05 FP8 GEMM."""

    def __init__(self, weight: torch.Tensor, bias: Optional[torch.Tensor], layer_prec: LayerPrecision) -> None:
        super().__init__()
        self.layer_prec = layer_prec
        self.register_buffer("weight", weight)
        self.register_buffer("bias", bias if bias is not None else torch.empty(0))
        self._has_bias = bias is not None
        self._w_fp8: Optional[torch.Tensor] = None
        self._w_scale: Optional[torch.Tensor] = None
        self._bias16: Optional[torch.Tensor] = None
        if layer_prec.weight.is_fp8():
            self._quantise_weights()

    def _quantise_weights(self) -> None:
        dev = self.weight.device if self.weight.is_cuda else torch.device("cuda")
        w16 = self.weight.detach().to(dev, torch.float16).contiguous()
        self._w_fp8, self._w_scale = ops.quantise(w16, self.layer_prec.weight.fmt())
        if self._has_bias:
            self._bias16 = self.bias.detach().to(dev, torch.float16).contiguous()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not self.layer_prec.is_fp8():
            return nn.functional.linear(x, self.weight, self.bias if self._has_bias else None)
        act = self.layer_prec.activation
        afmt = act.fmt() if act.is_fp8() else "e4m3"
        wfmt = self.layer_prec.weight.fmt() if self.layer_prec.weight.is_fp8() else "e4m3"
        if self._w_fp8 is None:
            self._quantise_weights_as(wfmt)
        # quantise(x) then the scaled GEMM; one kernel for short M (decoder steps)
        out, _, _ = ops.linear_fp8(x.half().contiguous(), self._w_fp8, self._w_scale, self._bias16, a_format=afmt,
                                   w_format=wfmt)
        return out

    def _quantise_weights_as(self, fmt: str) -> None:
        w16 = self.weight.detach().to("cuda", torch.float16).contiguous()
        self._w_fp8, self._w_scale = ops.quantise(w16, fmt)
        if self._has_bias:
            self._bias16 = self.bias.detach().to(w16.device, torch.float16).contiguous()


class BlazeLayerNorm(nn.Module):
    """Drop-in nn.LayerNorm backed by the fused CUDA kernel."""

    VECTOR_WIDTH = 8

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor, eps: float = 1e-5) -> None:
        super().__init__()
        self.register_buffer("weight", weight)
        self.register_buffer("bias", bias)
        self.eps = eps

    @classmethod
    def supports(cls, ln: nn.LayerNorm) -> bool:
        return (len(ln.normalized_shape) == 1 and ln.normalized_shape[0] % cls.VECTOR_WIDTH == 0
                and ln.elementwise_affine and ln.bias is not None)

    @classmethod
    def from_layernorm(cls, ln: nn.LayerNorm) -> "BlazeLayerNorm":
        return cls(ln.weight.data.detach().half().contiguous(), ln.bias.data.detach().half().contiguous(), ln.eps)

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        if (x.is_cuda and x.dtype == torch.float16 and x.is_contiguous() and x.size(-1) % self.VECTOR_WIDTH == 0
                and (residual is None or (residual.is_contiguous() and residual.dtype == torch.float16))):
            return ops.layernorm(x, residual, self.weight, self.bias, self.eps)[0]
        hidden = x if residual is None else x + residual
        return nn.functional.layer_norm(hidden, [hidden.size(-1)], self.weight.to(hidden.dtype),
                                        self.bias.to(hidden.dtype), self.eps)
