"""CPU reference of the FP8 Whisper encoder stack + CPU timing harness (test infrastructure only).

Structure: HF WhisperEncoderLayer (transformers 5.5.0,
models/whisper/modeling_whisper.py:361-415): pre-LN self-attention block and
FFN block with residual adds, exact-erf GELU, and the fp16 clamp at the end of
the layer; a final LayerNorm after the last layer (WhisperEncoder.layer_norm).
Every linear is the reference's FP8 linear semantics
(whisper_blaze/model.py:80-109): per-tensor E4M3 quantise of the activation
and of the weight, fp32 matmul of the dequantised operands, bias. Attention is
torch SDPA in fp32 on the CPU.

Rounding points follow the B200 stack (fp16 storage between ops; the residual
adds are fused into the linear's fp32 epilogue and rounded once; GELU applies
to the fp16 fc1 output and is rounded to fp16, as in HF), so the two are
compared with relative-error gates rather than bit for bit.

This is also the path `bench.py --impl reference` and the `cpu_baseline` leg
time: torch-CPU fp32 dequantise + matmul on all host cores.
"""
from __future__ import annotations

import os
import time

import numpy as np
import torch
import torch.nn.functional as F

from . import fp8, gemm, norm


def _q(t16: torch.Tensor):
    q, s = fp8.quantise_torch(t16, fp8.E4M3)
    return q, float(s)


def quantise_layer(lw) -> dict:
    """Quantise one layer's fp16 master weights (attributes as in LayerWeights)."""
    out = {}
    for name in ("w_qkv", "w_o", "w_fc1", "w_fc2"):
        out[name] = _q(getattr(lw, name).cpu())
    for name in ("ln1_g", "ln1_b", "b_qkv", "b_o", "ln2_g", "ln2_b", "b_fc1", "b_fc2"):
        out[name] = getattr(lw, name).cpu()
    return out


def _linear(x16: torch.Tensor, w, bias, residual=None, epilogue=gemm.EPI_NONE) -> torch.Tensor:
    xq, sx = _q(x16)
    wq, sw = w
    return gemm.gemm_fp8_ref(xq, sx, wq, sw, bias, residual, epilogue)


def encoder_layer_ref(h: torch.Tensor, qw: dict, B: int, S: int, heads: int, eps: float = 1e-5) -> torch.Tensor:
    """h [B*S, D] fp16 (CPU) -> next hidden state [B*S, D] fp16."""
    T, D = h.shape
    Dh = D // heads
    x = norm.layernorm_ref(h, None, qw["ln1_g"], qw["ln1_b"], eps).half()
    qkv = _linear(x, qw["w_qkv"], qw["b_qkv"])
    q, k, v = (qkv.float().view(B, S, 3, heads, Dh)[:, :, i].transpose(1, 2) for i in range(3))
    a = F.scaled_dot_product_attention(q, k, v).transpose(1, 2).reshape(T, D).half()
    h2 = _linear(a, qw["w_o"], qw["b_o"], residual=h, epilogue=gemm.EPI_RESIDUAL)
    x2 = norm.layernorm_ref(h2, None, qw["ln2_g"], qw["ln2_b"], eps).half()
    y = _linear(x2, qw["w_fc1"], qw["b_fc1"])          # fc1 output, fp16
    f = gemm.gelu_f16(y)                                 # GELU on the fp16 output, rounded to fp16 (HF order)
    return _linear(f, qw["w_fc2"], qw["b_fc2"], residual=h2, epilogue=gemm.EPI_RESIDUAL_CLAMP)


def encoder_stack_ref(hidden: torch.Tensor, qlayers: list, heads: int, final_ln=None,
                      eps: float = 1e-5) -> torch.Tensor:
    """hidden [B, S, D] fp16 -> [B, S, D] fp16 after all layers and the final LayerNorm."""
    B, S, D = hidden.shape
    h = hidden.cpu().reshape(B * S, D)
    for qw in qlayers:
        h = encoder_layer_ref(h, qw, B, S, heads, eps)
    g, b = final_ln if final_ln is not None else (torch.ones(D, dtype=torch.float16),
                                                  torch.zeros(D, dtype=torch.float16))
    return norm.layernorm_ref(h, None, g, b, eps).half().view(B, S, D)


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def time_cpu_chunk(qlayers: list, seq_len: int, d_model: int, heads: int, n_layers_total: int,
                   budget_s: float = 20.0, seed: int = 0) -> dict:
    """Time one chunk [1, seq_len, d_model] through the CPU reference stack.

    Runs layers until all `n_layers_total` are done or `budget_s` is spent
    (at least one), then extrapolates the per-layer average to the full
    stack. Returns chunks/s, the layers actually run and the threads used.
    """
    threads = host_threads()
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(seed)
    h = torch.randn(seq_len, d_model, generator=g).half()
    done = 0
    t0 = time.perf_counter()
    while done < n_layers_total:
        h = encoder_layer_ref(h, qlayers[done % len(qlayers)], 1, seq_len, heads)
        done += 1
        if time.perf_counter() - t0 > budget_s:
            break
    per_layer = (time.perf_counter() - t0) / done
    chunk_s = per_layer * n_layers_total
    return {"chunks_per_s": 1.0 / chunk_s, "chunk_seconds": chunk_s, "layers_run": done,
            "layers_total": n_layers_total, "threads": threads}
