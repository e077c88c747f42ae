"""nn.Module equivalents of the reference's BlazeLinear and BlazeLayerNorm.

BlazeLinear mirrors whisper_blaze/model.py:47-109 (same constructor, buffers
and FP16 path) but its FP8 branch runs the B200 FP8 GEMM on the quantised
operands instead of dequantising both and calling an fp16 F.linear; the
weight is quantised once at construction and its scale stays on the device.
BlazeLayerNorm mirrors model.py:116-168 unchanged in behaviour.
"""
from __future__ import annotations

import weakref
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

    def _quantise_weights(self, fmt: Optional[str] = None) -> None:
        """Quantise the fp16 weight once (format `fmt`, default the weight precision's) and
        keep its codes, device scale and fp16 bias on the weight's GPU (the current one if
        the weight is on the host)."""
        dev = self.weight.device if self.weight.is_cuda else torch.device("cuda")
        w16 = self.weight.detach().to(dev, torch.float16).contiguous()
        self._w_fp8, self._w_scale = ops.quantise(w16, fmt or self.layer_prec.weight.fmt())
        if self._has_bias:
            self._bias16 = self.bias.detach().to(dev, torch.float16).contiguous()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not self.layer_prec.is_fp8():
            return nn.functional.linear(x, self.weight, self.bias if self._has_bias else None)
        act = self.layer_prec.activation
        afmt = act.fmt() if act.is_fp8() else "e4m3"
        wfmt = self.layer_prec.weight.fmt() if self.layer_prec.weight.is_fp8() else "e4m3"
        if self._w_fp8 is None:
            self._quantise_weights(wfmt)
        # quantise(x) then the scaled GEMM; one kernel for short M (decoder steps)
        out, _, _ = ops.linear_fp8(x.half().contiguous(), self._w_fp8, self._w_scale, self._bias16, a_format=afmt,
                                   w_format=wfmt)
        return out


class StackedKVProjection(nn.Module):
    """A cross-attention layer's k_proj and v_proj as ONE FP8 linear.

    The decoder's cross-attention projects the same encoder states twice, once
    per generate call per layer. Here the two weights are stacked into one
    [N_k + N_v, K] FP8 weight with one per-tensor scale (the stacked K/V shape
    of config 4), and `half(0)` / `half(1)` are drop-in modules for k_proj and
    v_proj: the first of them called on an input tensor runs the GEMM, the
    other returns its half of the cached output (a strided view) if called on
    the same, unmodified tensor; the cache is dropped once both halves were
    served. Mirrors the two separate projections of HF's WhisperAttention
    (cross-attention branch), whose results the stacked GEMM reproduces up to
    the shared weight scale.
    """

    def __init__(self, k_proj: nn.Linear, v_proj: nn.Linear, layer_prec: LayerPrecision) -> None:
        super().__init__()
        if k_proj.in_features != v_proj.in_features:
            raise ValueError("k_proj and v_proj must read the same input width")
        self.n_k = k_proj.out_features
        w = torch.cat([k_proj.weight.data.detach(), v_proj.weight.data.detach()], dim=0)
        biases = []
        for lin in (k_proj, v_proj):
            biases.append(lin.bias.data.detach() if lin.bias is not None
                          else torch.zeros(lin.out_features, dtype=lin.weight.dtype, device=lin.weight.device))
        self.linear = BlazeLinear(w, torch.cat(biases), layer_prec)
        self._cache = None  # (weakref to input, input version, output, halves served bitmask)

    def project(self, x: torch.Tensor, which: int) -> torch.Tensor:
        ent = self._cache
        if ent is not None and ent[0]() is x and ent[1] == x._version:
            out, served = ent[2], ent[3]
        else:
            out, served = self.linear(x), 0
        served |= 1 << which
        self._cache = None if served == 3 else (weakref.ref(x), x._version, out, served)
        return out[..., :self.n_k] if which == 0 else out[..., self.n_k:]

    def half(self, which: int) -> "StackedKVHalf":
        return StackedKVHalf(self, which)


class StackedKVHalf(nn.Module):
    """k_proj (which=0) or v_proj (which=1) of a StackedKVProjection."""

    def __init__(self, stacked: StackedKVProjection, which: int) -> None:
        super().__init__()
        object.__setattr__(self, "_stacked", stacked)  # owned (registered) by the attention module
        self.which = which

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self._stacked.project(x, self.which)


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
