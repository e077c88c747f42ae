"""Whisper-large-v3-shaped encoder stack with every linear in FP8 E4M3.

Layer structure is HF WhisperEncoderLayer (pre-LN): LN -> self-attention ->
+residual -> LN -> fc1 -> GELU(erf) -> fc2 -> +residual -> fp16 clamp, then a
final LayerNorm after the last layer. q/k/v are one fused [3*D, D] projection
(k has no bias, so its third of the bias is zero). Attention runs in fp16 with
fp32 softmax on the tcgen05 attention kernel (ops.attention) straight from the
strided q/k/v views, which also reports max|out|; torch SDPA (what HF runs in
the reference) is selectable for comparison.

Per layer, on one stream and without any host synchronisation:

  LN1(h) -> fp8     -> xq  (fp8)  + scale              norm stats pass + norm quantise pass
                                                       (the fp16 LN output is never stored)
  QKV GEMM          -> qkv (fp16), bias epilogue       tcgen05 GEMM
  attention(q,k,v)  -> a   (fp16) + max|a|             tcgen05 attention kernel
  quantise(a)       -> aq  (fp8)
  out-proj GEMM     -> h2 = fp16(acc*s + b + h)        residual epilogue
  LN2(h2) -> fp8    -> x2q                             norm stats pass + norm quantise pass
  fc1 GEMM          -> y = fp16(acc*s + b) + max(y)          bias + max-key epilogue
  gelu+quantise(y)  -> fq = q8(fp16(gelu(y)))              (amax of the GELU output from max(y))
  fc2 GEMM          -> h' = fp16(clamp(acc*s + b + h2))      residual+clamp epilogue

Activation scales live in device memory; weights are quantised once.
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field
from typing import Callable, List, Optional, Sequence

import torch
import torch.nn.functional as F

from . import ops


@dataclass
class EncoderConfig:
    d_model: int = 1280
    heads: int = 20
    ffn: int = 5120
    layers: int = 32
    seq_len: int = 1500
    eps: float = 1e-5

    @property
    def head_dim(self) -> int:
        return self.d_model // self.heads

    def gemm_flops_per_token(self) -> int:
        """FP8 GEMM FLOPs per token per layer (QKV + out-proj + fc1 + fc2)."""
        D, Fd = self.d_model, self.ffn
        return 2 * D * (3 * D + D + Fd) + 2 * Fd * D

    def attn_flops_per_chunk(self) -> int:
        """fp16 attention FLOPs per chunk per layer (QK^T and PV)."""
        return 4 * self.seq_len * self.seq_len * self.d_model


@dataclass
class LayerWeights:
    """fp16 master weights of one encoder layer (nn.Linear layout [out, in])."""
    ln1_g: torch.Tensor
    ln1_b: torch.Tensor
    w_qkv: torch.Tensor
    b_qkv: torch.Tensor
    w_o: torch.Tensor
    b_o: torch.Tensor
    ln2_g: torch.Tensor
    ln2_b: torch.Tensor
    w_fc1: torch.Tensor
    b_fc1: torch.Tensor
    w_fc2: torch.Tensor
    b_fc2: torch.Tensor

    def to(self, device) -> "LayerWeights":
        return LayerWeights(**{k: v.to(device) for k, v in self.__dict__.items()})


def random_layer_weights(cfg: EncoderConfig, gen: torch.Generator, std: float = 0.02) -> LayerWeights:
    """Random-init weights on the CPU: linears and biases ~ N(0, std), k bias 0, LN gamma 1 beta 0."""
    D, Fd = cfg.d_model, cfg.ffn

    def n(*shape):
        return (torch.randn(*shape, generator=gen, dtype=torch.float32) * std).half()

    b_qkv = n(3 * D)
    b_qkv[D:2 * D] = 0  # k_proj has no bias
    return LayerWeights(
        ln1_g=torch.ones(D, dtype=torch.float16), ln1_b=torch.zeros(D, dtype=torch.float16),
        w_qkv=n(3 * D, D), b_qkv=b_qkv, w_o=n(D, D), b_o=n(D),
        ln2_g=torch.ones(D, dtype=torch.float16), ln2_b=torch.zeros(D, dtype=torch.float16),
        w_fc1=n(Fd, D), b_fc1=n(Fd), w_fc2=n(D, Fd), b_fc2=n(D))


def synthetic_stack_weights(cfg: EncoderConfig, device, seed: int = 1234, std: float = 0.02) -> List[LayerWeights]:
    """The benchmark's random-init weights: cfg.layers layers drawn in order on `device` from one
    seeded generator (linears and biases ~ N(0, std), k bias 0, LN gamma 1 beta 0), so every
    process that calls this with the same arguments holds the same bits."""
    dev = torch.device(device)
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    D, Fd = cfg.d_model, cfg.ffn

    def n(*shape):
        return (torch.randn(*shape, generator=gen, device=dev, dtype=torch.float32) * std).half()

    def const(v):
        return torch.full((D,), v, dtype=torch.float16, device=dev)

    layers = []
    for _ in range(cfg.layers):
        b_qkv = n(3 * D)
        b_qkv[D:2 * D] = 0  # k_proj has no bias
        layers.append(LayerWeights(ln1_g=const(1.0), ln1_b=const(0.0), w_qkv=n(3 * D, D), b_qkv=b_qkv,
                                   w_o=n(D, D), b_o=n(D), ln2_g=const(1.0), ln2_b=const(0.0),
                                   w_fc1=n(Fd, D), b_fc1=n(Fd), w_fc2=n(D, Fd), b_fc2=n(D)))
    return layers


def synthetic_hidden(chunks: int, cfg: EncoderConfig, device, seed: int) -> torch.Tensor:
    """The benchmark's input shard: [chunks, seq_len, d_model] fp16 ~ N(0, 1), drawn on `device`
    from a generator seeded with `seed` (the benchmark uses 99 + rank)."""
    dev = torch.device(device)
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    return torch.randn(chunks, cfg.seq_len, cfg.d_model, generator=gen, device=dev, dtype=torch.float32).half()


@dataclass
class _QuantLayer:
    ln1_g: torch.Tensor
    ln1_b: torch.Tensor
    w_qkv: torch.Tensor
    s_qkv: torch.Tensor
    b_qkv: torch.Tensor
    w_o: torch.Tensor
    s_o: torch.Tensor
    b_o: torch.Tensor
    ln2_g: torch.Tensor
    ln2_b: torch.Tensor
    w_fc1: torch.Tensor
    s_fc1: torch.Tensor
    b_fc1: torch.Tensor
    w_fc2: torch.Tensor
    s_fc2: torch.Tensor
    b_fc2: torch.Tensor


@dataclass
class GemmTiming:
    """CUDA-event bracket around one GEMM launch (for roofline accounting)."""
    start: torch.cuda.Event
    end: torch.cuda.Event
    flops: int
    name: str = ""

    def ms(self) -> float:
        return self.start.elapsed_time(self.end)


class FP8EncoderStack:
    """Encoder stack on one GPU. forward() takes [B, S, D] fp16 on the device."""

    def __init__(self, cfg: EncoderConfig, layers: List[LayerWeights], device,
                 final_ln: Optional[tuple] = None, slice_chunks: Optional[int] = None,
                 attention: Optional[str] = None) -> None:
        """slice_chunks: run the batch through the whole stack this many chunks at a
        time (None = all at once). Smaller slices keep each slice's [tokens, d_model]
        tensors (1500 x 1280 x 2 B = 3.84 MB per chunk) inside the 126 MB L2, so the
        passes that read a tensor twice (LayerNorm statistics then quantise,
        amax then quantise) hit L2 on the second read.

        attention: "sdpa" (default; torch SDPA, cuDNN on B200, then an amax
        pass) or "wbk" (the tcgen05 attention kernel, which also emits
        max|out| for the following quantise); the WBK_ATTENTION environment
        variable sets the default."""
        self.cfg = cfg
        self.attention = attention or os.environ.get("WBK_ATTENTION", "sdpa")
        if self.attention not in ("wbk", "sdpa"):
            raise ValueError(f"attention must be 'wbk' or 'sdpa', not {self.attention!r}")
        self.slice_chunks = slice_chunks
        self.device = torch.device(device)
        self.layers: List[_QuantLayer] = []
        with torch.cuda.device(self.device):
            for lw in layers:
                lw = lw.to(self.device)
                wq, sq = ops.quantise(lw.w_qkv.contiguous())
                wo, so = ops.quantise(lw.w_o.contiguous())
                w1, s1 = ops.quantise(lw.w_fc1.contiguous())
                w2, s2 = ops.quantise(lw.w_fc2.contiguous())
                self.layers.append(_QuantLayer(lw.ln1_g, lw.ln1_b, wq, sq, lw.b_qkv, wo, so, lw.b_o,
                                               lw.ln2_g, lw.ln2_b, w1, s1, lw.b_fc1, w2, s2, lw.b_fc2))
            D = cfg.d_model
            if final_ln is None:
                final_ln = (torch.ones(D, dtype=torch.float16), torch.zeros(D, dtype=torch.float16))
            self.final_g = final_ln[0].to(self.device)
            self.final_b = final_ln[1].to(self.device)
        self._ws_tokens = -1
        self.gemm_timings: Optional[List[GemmTiming]] = None  # set to [] to record
        self.launches_per_forward: Optional[int] = None  # libwbk launches of the last eager forward
        self._graphs: dict = {}  # (input, shape, device, output) -> (CUDA graph, output tensor)
        self._stream_state = None
        self._host_in = None

    # -------------------------------------------------------------- buffers
    def _workspace(self, T: int) -> None:
        if self._ws_tokens == T:
            return
        self._graphs.clear()  # captured graphs point into the buffers being replaced
        D, Fd, dev = self.cfg.d_model, self.cfg.ffn, self.device
        e = lambda *s, dt=torch.float16: torch.empty(*s, dtype=dt, device=dev)  # noqa: E731
        self.h_a, self.h_b, self.h2 = e(T, D), e(T, D), e(T, D)
        self.x, self.attn = e(T, D), e(T, D)
        self.xq, self.aq = e(T, D, dt=torch.uint8), e(T, D, dt=torch.uint8)
        self.qkv = e(T, 3 * D)
        self.f = e(T, Fd)
        self.fq = e(T, Fd, dt=torch.uint8)
        self.out = e(T, D)
        self.amax = torch.zeros(8, dtype=torch.int32, device=dev)
        self.ln_ws = ops.layernorm_quantise_ws(T, dev)
        self.scales = torch.ones(4, dtype=torch.float32, device=dev)
        self._ws_tokens = T

    def _gemm(self, name: str, flops: int, *args, **kwargs) -> torch.Tensor:
        if self.gemm_timings is None:
            return ops.gemm_fp8(*args, **kwargs)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        out = ops.gemm_fp8(*args, **kwargs)
        e.record()
        self.gemm_timings.append(GemmTiming(s, e, flops, name))
        return out

    # -------------------------------------------------------------- compute
    def _attention(self, qkv_buf: torch.Tensor, attn_buf: torch.Tensor, B: int, S: int,
                   amax_ws: torch.Tensor) -> torch.Tensor:
        """Self-attention on the strided q/k/v views of the fused QKV output -> [T, D] fp16,
        with max|out| max-accumulated into amax_ws."""
        cfg = self.cfg
        H, Dh = cfg.heads, cfg.head_dim
        qkv = qkv_buf.view(B, S, 3, H, Dh)
        q, k, v = (qkv[:, :, i].transpose(1, 2) for i in range(3))
        if self.attention == "wbk":
            ops.attention(q, k, v, out=attn_buf.view(B, S, H, Dh).transpose(1, 2), out_amax=amax_ws)
            return attn_buf
        o = F.scaled_dot_product_attention(q, k, v)  # [B, H, S, Dh]
        o = o.transpose(1, 2)
        if o.is_contiguous():
            o = o.reshape(B * S, cfg.d_model)
        else:
            attn_buf.view(B, S, H, Dh).copy_(o)
            o = attn_buf
        ops.amax_accumulate(o, amax_ws)
        return o

    def _layer(self, L: _QuantLayer, h: torch.Tensor, h_next: torch.Tensor, B: int, S: int,
               capture: Optional[dict] = None) -> None:
        cfg = self.cfg
        T, D, Fd = B * S, cfg.d_model, cfg.ffn
        amax, sc = self.amax, self.scales
        keep = (lambda k, t: capture.__setitem__(k, t.clone())) if capture is not None else (lambda k, t: None)
        # row views of the workspace for this slice (T <= the rows the workspace was sized for)
        xq, aq, qkv, h2, f, fq, attn_buf = (b[:T] for b in (self.xq, self.aq, self.qkv, self.h2, self.f, self.fq,
                                                             self.attn))
        amax.zero_()
        ops.layernorm_quantise(h, L.ln1_g, L.ln1_b, cfg.eps, q_out=xq, scale_out=sc[0:1], ws=self.ln_ws,
                               amax_ws=amax[0:1])
        if capture is not None:
            keep("ln1", ops.layernorm(h, None, L.ln1_g, L.ln1_b, cfg.eps)[0])
        keep("ln1_q", xq), keep("ln1_s", sc[0:1])
        self._gemm("qkv", 2 * T * D * 3 * D, xq, sc[0:1], L.w_qkv, L.s_qkv, L.b_qkv, out=qkv)
        keep("qkv", qkv)
        attn = self._attention(qkv, attn_buf, B, S, amax[1:2])
        ops.quantise_from_amax(attn, amax[1:2], q_out=aq, scale_out=sc[1:2])
        keep("attn", attn), keep("attn_q", aq), keep("attn_s", sc[1:2])
        self._gemm("out_proj", 2 * T * D * D, aq, sc[1:2], L.w_o, L.s_o, L.b_o, residual=h,
                   epilogue="residual", out=h2)
        keep("h2", h2)
        ops.layernorm_quantise(h2, L.ln2_g, L.ln2_b, cfg.eps, q_out=xq, scale_out=sc[2:3],
                               ws=self.ln_ws, amax_ws=amax[2:3])
        if capture is not None:
            keep("ln2", ops.layernorm(h2, None, L.ln2_g, L.ln2_b, cfg.eps)[0])
        keep("ln2_q", xq), keep("ln2_s", sc[2:3])
        self._gemm("fc1", 2 * T * D * Fd, xq, sc[2:3], L.w_fc1, L.s_fc1, L.b_fc1, epilogue="bias_maxkey",
                   out=f, out_amax=amax[3:4])
        ops.quantise_gelu(f, amax[3:4], q_out=fq, scale_out=sc[3:4], amax_ws=amax[4:5])
        keep("fc1", f), keep("fc1_q", fq), keep("fc1_s", sc[3:4])
        self._gemm("fc2", 2 * T * Fd * D, fq, sc[3:4], L.w_fc2, L.s_fc2, L.b_fc2, residual=h2,
                   epilogue="residual_clamp", out=h_next)
        keep("out", h_next)

    @torch.inference_mode()
    def forward(self, hidden: torch.Tensor, out: Optional[torch.Tensor] = None,
                capture: Optional[List[dict]] = None,
                capture_layers: Optional[Sequence[int]] = None) -> torch.Tensor:
        """hidden [B, S, D] fp16 on this stack's device -> [B, S, D] fp16 (the final LayerNorm applied).

        capture: if a list is given, one dict per layer of copies of that
        layer's intermediates (LN outputs, fp8 codes and scales, qkv,
        attention, fc1, residual sums; "layer" holds the layer index) is
        appended — for stage-wise parity checks; it costs copies, so it is off
        on the production path. capture_layers restricts it to those layer
        indices (the copies of one full-batch layer take about 4 GB)."""
        ops.require_input(hidden, "hidden")
        ops.require_fp16(hidden, "hidden")
        B, S, D = hidden.shape
        if D != self.cfg.d_model:
            raise RuntimeError(f"hidden size {D} != d_model {self.cfg.d_model}")
        step = B if not self.slice_chunks else min(B, self.slice_chunks)
        launches0 = ops.LAUNCHES[0]
        with torch.cuda.device(self.device):
            self._workspace(step * S)
            if out is None:
                if step == B:
                    o_full = self.out
                else:
                    o_full = torch.empty(B * S, D, dtype=torch.float16, device=self.device)
            else:
                o_full = out.view(B * S, D)
            for b0 in range(0, B, step):
                nb = min(step, B - b0)
                T = nb * S
                h = hidden[b0:b0 + nb].reshape(T, D)
                bufs = (self.h_a[:T], self.h_b[:T])
                for i, L in enumerate(self.layers):
                    nxt = bufs[i % 2]
                    cap = None
                    if capture is not None and (capture_layers is None or i in capture_layers):
                        cap = {"in": h.clone(), "layer": i}
                        capture.append(cap)
                    self._layer(L, h, nxt, nb, S, cap)
                    h = nxt
                ops.layernorm(h, None, self.final_g, self.final_b, self.cfg.eps, out=o_full[b0 * S:b0 * S + T])
        self.launches_per_forward = ops.LAUNCHES[0] - launches0
        return o_full.view(B, S, D)

    @torch.inference_mode()
    def forward_graphed(self, hidden: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """forward() replayed from a CUDA graph: the ~36 launches per layer cost one
        graph launch. A graph is captured on the first call for a given (input,
        output) pair of tensors (addresses and shape) and replayed on later calls
        with the same tensors; with out=None the result lives in the stack's own
        output buffer and is overwritten by the next replay."""
        ops.require_input(hidden, "hidden")
        key = (hidden.data_ptr(), tuple(hidden.shape), hidden.device, None if out is None else out.data_ptr())
        entry = self._graphs.get(key)
        if entry is None:
            with torch.cuda.device(self.device):
                self.forward(hidden, out=out)  # sizes the workspace and runs every lazy initialisation
                torch.cuda.synchronize(self.device)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    y = self.forward(hidden, out=out)
                torch.cuda.synchronize(self.device)
            entry = (g, y)
            self._graphs[key] = entry
        entry[0].replay()
        return entry[1]

    @torch.inference_mode()
    def forward_host_stream(self, host_inputs: Sequence[torch.Tensor],
                            host_outputs: Sequence[Optional[torch.Tensor]],
                            post: Optional[Callable[[torch.Tensor], torch.Tensor]] = None) -> None:
        """Pipelined host-to-host inference over a sequence of pinned batches.

        Batch i's host->device copy runs on one copy stream and batch i-1's
        device->host copy on another while batch i-1 / i compute (graphed)
        on the current stream, through two device input and two device output
        buffers ordered by events; `post` (e.g. an all-gather of the sharded
        outputs) runs on the current stream after each forward and its result
        is what lands in host_outputs[i] (None entries skip the copy-out).
        Returns with every copy enqueued
        before the current stream's next work (the caller synchronises)."""
        if len(host_inputs) != len(host_outputs):
            raise ValueError("host_inputs and host_outputs must have the same length")
        if not host_inputs:
            return
        shape = tuple(host_inputs[0].shape)
        dev = self.device
        cs = torch.cuda.current_stream(dev)
        if self._stream_state is None or self._stream_state["shape"] != shape:
            e = lambda: torch.empty(shape, dtype=torch.float16, device=dev)  # noqa: E731
            self._stream_state = {"shape": shape, "in": [e(), e()], "out": [e(), e()],
                                  "h2d": torch.cuda.Stream(dev), "d2h": torch.cuda.Stream(dev)}
        st = self._stream_state
        h2d_s, d2h_s = st["h2d"], st["d2h"]
        ev_h2d = [torch.cuda.Event() for _ in range(2)]
        ev_comp = [torch.cuda.Event() for _ in range(2)]
        ev_d2h = [torch.cuda.Event() for _ in range(2)]
        with torch.cuda.device(dev):
            # the buffers may still be read or written by work queued before this call
            h2d_s.wait_stream(cs)
            d2h_s.wait_stream(cs)
            for i, (hin, hout) in enumerate(zip(host_inputs, host_outputs)):
                b = i % 2
                with torch.cuda.stream(h2d_s):
                    if i >= 2:
                        h2d_s.wait_event(ev_comp[b])  # forward i-2 has finished reading in[b]
                    st["in"][b].copy_(hin, non_blocking=True)
                    ev_h2d[b].record(h2d_s)
                cs.wait_event(ev_h2d[b])
                if i >= 2:
                    cs.wait_event(ev_d2h[b])  # copy-out of i-2 has finished reading out[b]
                y = self.forward_graphed(st["in"][b], out=st["out"][b])
                res = post(y) if post is not None else y
                ev_comp[b].record(cs)
                with torch.cuda.stream(d2h_s):
                    d2h_s.wait_event(ev_comp[b])
                    if hout is not None:  # None: this rank keeps no host copy
                        hout.copy_(res, non_blocking=True)
                    ev_d2h[b].record(d2h_s)
                if res is not y:
                    res.record_stream(d2h_s)
            cs.wait_stream(d2h_s)
            cs.wait_stream(h2d_s)

    def device_input(self, hidden_host: torch.Tensor) -> torch.Tensor:
        """Copy a (pinned) host batch into this stack's persistent device input buffer
        (asynchronously, on the current stream) and return that buffer — the same
        tensor every call, so a graphed forward on it is captured once."""
        if self._host_in is None or self._host_in.shape != hidden_host.shape:
            self._host_in = torch.empty(hidden_host.shape, dtype=torch.float16, device=self.device)
        self._host_in.copy_(hidden_host, non_blocking=True)
        return self._host_in

    @torch.inference_mode()
    def forward_host(self, hidden_host: torch.Tensor, out_host: Optional[torch.Tensor] = None,
                     graphed: bool = False) -> torch.Tensor:
        """Host-to-host call: copy in (from pinned memory), run, copy out."""
        dev_in = self.device_input(hidden_host)
        y = self.forward_graphed(dev_in) if graphed else self.forward(dev_in)
        if out_host is None:
            out_host = torch.empty(y.shape, dtype=y.dtype, pin_memory=True)
        out_host.copy_(y, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return out_host
