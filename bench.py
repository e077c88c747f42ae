"""Benchmark of the B200 FP8 quantised-matmul path (whisper-blaze north star).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload stack|layer|fc1|decoder|crossattn|attention|norms|fp8peak]

Default workload (config 5 of the north star): a 32-layer Whisper-large-v3
encoder stack (d_model 1280, 20 heads, FFN 5120, pre-LN, every linear FP8
E4M3 per-tensor scaled, fp16 torch-SDPA attention), random-init weights,
synthetic post-conv hidden states [64 chunks, 1500, 1280] fp16 ~ N(0,1).
The 64 chunks are split by batch over N GPUs (one process per GPU under
torchrun, NCCL), outputs gathered with one all_gather_into_tensor. A step is
one pass of the whole stack over the whole batch plus the gather; metric
chunks/s = 64 / max-over-ranks step time (strong scaling: total work fixed).

Prints ONE JSON line on rank 0. `value` has the inputs resident in HBM;
`e2e` is the same metric through the public host API (pinned host input ->
device, stack, gather, device -> host output on rank 0), copies timed, steps
streamed by FP8EncoderStack.forward_host_stream (step i's copy-in and step
i-1's copy-out overlap step i's compute).
`roofline` is for the dominant kernel (the tcgen05 FP8 GEMM): achieved
TFLOP/s = algorithmic FLOPs of the GEMM launches in the timed steps / their
CUDA-event time. `cpu_baseline` (rank 0, N = 1) and `--impl reference` time
the reference's CPU path (torch-CPU fp32 dequantise + matmul, oracle/encoder.py)
on one chunk on all host cores.

Secondary workloads print their own line with their
own metric: fc1 (config 1), layer (config 2), decoder (config 3), crossattn
(config 4); attention (the encoder self-attention kernel against torch SDPA)
and norms (the norm ops' HBM bandwidth) cover the other kernels; fp8peak
prints the measured dense FP8 ceiling alone (also measured, and used as
`roofline.peak`, in every stack run on rank 0).
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import time
import types

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [REPO, os.path.join(REPO, "whisper-blaze_b200")]

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

TOTAL_CHUNKS = 64
NOMINAL_FP8_TFLOPS = 4500.0


# ----------------------------------------------------------------- helpers

def measured_peaks() -> dict:
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"],
                "bf16_tflops_sustained": p.get("bf16_tflops_sustained", p["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def fp8_peak(sustained: bool) -> tuple[float, str]:
    p = measured_peaks()
    key = "bf16_tflops_sustained" if sustained else "bf16_tflops"
    return 2.0 * p[key], (f"2 x {key} of {p['source']} MEASURED_PEAKS.json "
                          f"(dense fp8 tensor rate is 2x dense bf16 on B200)")


def measure_fp8_peak(dev, seconds: float = 1.0, n: int = 8192) -> dict:
    """Dense FP8 tensor rate of this GPU, measured now the way MEASURED_PEAKS.json measures the
    bf16 one (a library GEMM): cuBLASLt's FP8 E4M3 GEMM (torch._scaled_mm, per-tensor fp32
    scales, bf16 out) on n x n x n operands -- best of 10 calls (burst) and back to back for
    `seconds` (sustained, under the power cap, SM clock sampled meanwhile). Our FP8 GEMM runs
    the same shape the same two ways, for comparison. TFLOP/s = 2 n^3 / t."""
    from whisper_blaze_b200 import ops
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    a = torch.randn(n, n, generator=g, device=dev).to(torch.float8_e4m3fn)
    b = torch.randn(n, n, generator=g, device=dev).to(torch.float8_e4m3fn)
    one = torch.ones((), dtype=torch.float32, device=dev)
    a8, b8 = a.view(torch.uint8), b.view(torch.uint8)
    out16 = torch.empty(n, n, dtype=torch.float16, device=dev)
    flops = 2.0 * n ** 3
    stream = torch.cuda.current_stream(dev)

    def lib_call():
        return torch._scaled_mm(a, b.t(), scale_a=one, scale_b=one, out_dtype=torch.bfloat16)

    def our_call():
        return ops.gemm_fp8(a8, one, b8, one, out=out16)

    def rates(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize(dev)
        best = float("inf")
        for _ in range(10):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            fn()
            e.record(stream)
            e.synchronize()
            best = min(best, s.elapsed_time(e))
        # sustained: enough back-to-back calls to fill `seconds` at the burst rate
        calls = max(10, int(seconds * 1e3 / best))
        with ClockSampler(dev.index) as clk:
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            for _ in range(calls):
                fn()
            e.record(stream)
            e.synchronize()
        c = clk.summary()
        return flops / best / 1e9, flops * calls / s.elapsed_time(e) / 1e9, c.get("sm_mhz"), c.get("reasons")

    lb, ls, lmhz, lreasons = rates(lib_call)
    ob, os_, omhz, _ = rates(our_call)
    return {"shape": f"{n}x{n}x{n} e4m3", "cublaslt_fp8_tflops_burst": lb, "cublaslt_fp8_tflops_sustained": ls,
            "cublaslt_sustained_sm_mhz": lmhz, "cublaslt_sustained_reasons": lreasons,
            "ours_tflops_burst": ob, "ours_tflops_sustained": os_, "ours_sustained_sm_mhz": omhz,
            "method": "torch._scaled_mm (cuBLASLt) and ops.gemm_fp8 on the same operands; best of 10 calls "
                      f"and {seconds:.1f} s back to back, CUDA events, NVML clocks"}


class ClockSampler:
    """SM clock, power and clock-event (throttle) reasons of this rank's GPU, sampled every
    10 ms through NVML on a background thread while the timed region runs (read-only queries);
    falls back to `nvidia-smi -lms 200` when NVML is unavailable."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.thread = None
        self.rows = []  # (sm_mhz, max_mhz, power_w, reason names)
        self.path = os.path.join("/tmp", f"wbk_clocks_{os.getpid()}.csv")

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        uuid = str(torch.cuda.get_device_properties(self.gpu).uuid)
        return pynvml, pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)

    def _poll(self, nv, h):
        sm_id = nv.NVML_CLOCK_SM
        max_mhz = nv.nvmlDeviceGetMaxClockInfo(h, sm_id)
        masks = [(name, getattr(nv, attr)) for name, attr in self.REASONS]
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(h, sm_id)
                watts = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
                bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.rows.append((float(mhz), float(max_mhz), watts, [n for n, m in masks if bits & m]))
            except Exception:  # noqa: BLE001 - a failed query only loses a sample
                pass
            self._stop.wait(0.01)

    def __enter__(self):
        import threading
        try:
            nv, h = self._nvml_handle()
            self._stop = threading.Event()
            self.thread = threading.Thread(target=self._poll, args=(nv, h), daemon=True)
            self.thread.start()
            return self
        except Exception:  # noqa: BLE001 - fall back to nvidia-smi
            self.thread = None
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.thread is not None:
            self._stop.set()
            self.thread.join(5)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self) -> dict:
        if self.thread is not None:
            rows = self.rows
            src = "nvml 10 ms"
        else:
            rows = []
            if self.proc is not None and os.path.exists(self.path):
                names = [n for n, _ in self.REASONS]
                with open(self.path) as f:
                    for line in f:
                        parts = [p.strip() for p in line.split(",")]
                        if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                            pw = float(parts[3]) if parts[3].replace(".", "").isdigit() else 0.0
                            rows.append((float(parts[1]), float(parts[2]), pw,
                                         [names[i] for i in range(4) if parts[5 + i].lower() == "active"]))
            src = "nvidia-smi 200 ms"
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        reasons = sorted({n for r in rows for n in r[3]})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": rows[0][1], "reasons": reasons,
                "samples": len(rows), "power_w_max": max(r[2] for r in rows), "sampler": src}


def setup_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    return world, rank, local


def max_over_ranks(v: float, world: int, device) -> float:
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(v: float, world: int, device) -> float:
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def barrier(world: int):
    if world > 1:
        dist.barrier()


def roofline_traffic(kernel_key: str):
    """dram bytes per launch from a committed ncu capture summary, if any."""
    path = os.path.join(REPO, "profiles", "traffic.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f).get(kernel_key)
    return None


# ------------------------------------------------------------ CPU reference

def cpu_reference_chunk(cfg, layers_fp16, budget_s: float) -> dict:
    from oracle import encoder as ref_encoder
    qlayers = [ref_encoder.quantise_layer(lw) for lw in layers_fp16]
    return ref_encoder.time_cpu_chunk(qlayers, cfg.seq_len, cfg.d_model, cfg.heads, cfg.layers, budget_s=budget_s)


def cpu_linear_seconds(x16: torch.Tensor, wq: torch.Tensor, w_scale: float, bias, residual, epi: str) -> float:
    """Seconds of one call of the reference's CPU path for an FP8 linear on the host cores:
    quantise the fp16 activation, fp32-dequantise both operands, fp32 matmul + bias +
    epilogue, fp16 result (oracle/fp8.py, oracle/gemm.py). Operands are CPU tensors."""
    from oracle import fp8 as ref_fp8
    from oracle import gemm as ref_gemm
    epi_code = {"none": ref_gemm.EPI_NONE, "gelu": ref_gemm.EPI_GELU, "residual": ref_gemm.EPI_RESIDUAL,
                "residual_clamp": ref_gemm.EPI_RESIDUAL_CLAMP, "bias_maxkey": ref_gemm.EPI_NONE}[epi]
    t0 = time.perf_counter()
    aq, sa = ref_fp8.quantise_torch(x16)
    ref_gemm.gemm_fp8_ref_f32(aq, float(sa), wq, w_scale, bias, residual, epi_code).half()
    return time.perf_counter() - t0


def cpu_layers(cfg, n_distinct: int = 2):
    """Distinct random layers for the CPU path (cycled through the 32 layers: the
    arithmetic per layer does not depend on which random weights it holds)."""
    from whisper_blaze_b200.encoder import random_layer_weights
    g = torch.Generator().manual_seed(0)
    return [random_layer_weights(cfg, g) for _ in range(n_distinct)]


def run_reference_arm(args, world, rank):
    if rank != 0:
        return
    from whisper_blaze_b200.encoder import EncoderConfig
    cfg = EncoderConfig(layers=args.layers)
    layers = cpu_layers(cfg)
    budget = max(2.0, args.ref_step_budget)
    samples = []
    info = None
    for i in range(args.warmup + args.steps):
        info = cpu_reference_chunk(cfg, layers, budget)
        if i >= args.warmup:
            samples.append(info["chunk_seconds"])
    chunk_s = statistics.median(samples)
    v = 1.0 / chunk_s
    line = {
        "impl": "reference", "metric": "encoder chunks/s (32-layer FP8 Whisper-large-v3 encoder stack)",
        "value": v, "unit": "chunks/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": chunk_s * 1e3, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "fp32 (fp8 codes dequantised)", "data": "synthetic",
        "config": {"workload": "encoder_stack (config 5)", "global_batch": TOTAL_CHUNKS, "seq_len": cfg.seq_len,
                   "d_model": cfg.d_model, "layers": cfg.layers, "parallelism": "host cores"},
        "cpu_baseline": {"value": v, "unit": "chunks/s", "cores": info["threads"], "kind": "port",
                         "sample": f"1 chunk (1500 frames), {info['layers_run']} of {cfg.layers} layers per step "
                                   f"timed, per-layer mean extrapolated to {cfg.layers}; torch-CPU fp32 "
                                   f"dequantise+matmul (oracle/encoder.py)"},
        "e2e": {"value": v, "unit": "chunks/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------- stack (ours)

def run_stack(args, world, rank, local):
    from whisper_blaze_b200 import ops
    from whisper_blaze_b200.encoder import (EncoderConfig, FP8EncoderStack, synthetic_hidden,
                                            synthetic_stack_weights)
    from whisper_blaze_b200.sharding import gather_batch, shard_bounds

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    cfg = EncoderConfig(layers=args.layers)
    D, Fd = cfg.d_model, cfg.ffn

    # random-init weights, generated on the device from a seeded generator (identical on every rank)
    layers = synthetic_stack_weights(cfg, dev, seed=1234)
    stack = FP8EncoderStack(cfg, layers, dev, slice_chunks=args.slice_chunks or None)
    del layers

    start, stop = shard_bounds(TOTAL_CHUNKS, world, rank)
    local_b = stop - start
    x = synthetic_hidden(local_b, cfg, dev, seed=99 + rank)

    def step():
        y = stack.forward_graphed(x) if args.graph else stack.forward(x)
        if world > 1:
            return gather_batch(y, TOTAL_CHUNKS)
        return y

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)

    stream = torch.cuda.current_stream(dev)
    launches0 = ops.LAUNCHES[0]
    if not args.graph:
        stack.gemm_timings = []
    with ClockSampler(local) as clocks:
        barrier(world)
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStart()  # profiler capture window = timed steps (no-op unprofiled)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(args.steps):
            step()
        t1.record(stream)
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
        barrier(world)
    launches = ops.LAUNCHES[0] - launches0
    if args.graph:
        # a replay issues the captured launches without passing through Python: count one eager step's
        launches = (stack.launches_per_forward or 0) * args.steps
    ms_local = t0.elapsed_time(t1) / args.steps
    ms = max_over_ranks(ms_local, world, dev)
    roofline_steps = args.steps
    if args.graph:
        # Kernel-level timing for the roofline: CUDA events bracket every GEMM launch of
        # eager steps run right after the timed graph replays (same kernels, same shapes).
        roofline_steps = max(1, min(args.steps, 3))
        stack.gemm_timings = []
        for _ in range(roofline_steps):
            stack.forward(x)
        torch.cuda.synchronize()
    gemm_ms = sum(t.ms() for t in stack.gemm_timings)
    gemm_flops = sum(t.flops for t in stack.gemm_timings)
    n_gemm = len(stack.gemm_timings)
    breakdown = {}
    for t in stack.gemm_timings:
        b = breakdown.setdefault(t.name, {"ms": 0.0, "flops": 0.0})
        b["ms"] += t.ms()
        b["flops"] += t.flops
    breakdown = {k: {"ms_per_step": v["ms"] / roofline_steps, "tflops": v["flops"] / (v["ms"] * 1e-3) / 1e12}
                 for k, v in breakdown.items()}
    stack.gemm_timings = None
    clock_info = clocks.summary()

    # e2e through the public host API: pinned host shard in, full output on rank 0's host out
    x_host = x.cpu().pin_memory()
    out_host = torch.empty((TOTAL_CHUNKS, cfg.seq_len, D), dtype=torch.float16, pin_memory=True) if rank == 0 else None
    e2e_steps = max(2, min(args.steps, 8))

    # Streaming host API: step i's copy-in and step i-1's copy-out overlap step i's compute.
    sink = out_host if rank == 0 else None  # only rank 0 copies the gathered output back
    post = (lambda y: gather_batch(y, TOTAL_CHUNKS)) if world > 1 else None  # noqa: E731

    def e2e_run(n):
        if args.graph:
            stack.forward_host_stream([x_host] * n, [sink] * n, post=post)
        else:
            for _ in range(n):
                y = stack.forward(stack.device_input(x_host))
                full = post(y) if post else y
                if sink is not None:
                    sink.copy_(full, non_blocking=True)

    e2e_run(2)  # captures the graphs of both buffer pairs
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    e2e_run(e2e_steps)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps, world, dev)
    h2d = sum_over_ranks(float(x_host.numel() * 2), world, dev)
    d2h = TOTAL_CHUNKS * cfg.seq_len * D * 2

    multi = None
    if world > 1:
        # The gather alone (device time, max over ranks), then a bitwise check on rank 0: each
        # rank's slice of the gathered output equals this process's own forward of that rank's
        # shard, regenerated from its seed. Activation scales are per rank's local batch.
        y = stack.forward_graphed(x)
        torch.cuda.synchronize()
        barrier(world)
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        full = gather_batch(y, TOTAL_CHUNKS)
        g1.record(stream)
        torch.cuda.synchronize()
        gather_ms = max_over_ranks(g0.elapsed_time(g1), world, dev)
        check = None
        if rank == 0:
            bad = []
            for r in range(world):
                s, e = shard_bounds(TOTAL_CHUNKS, world, r)
                yr = stack.forward(synthetic_hidden(e - s, cfg, dev, seed=99 + r))
                if not torch.equal(full[s:e], yr):
                    bad.append(r)
            check = "bit-identical" if not bad else f"MISMATCH on ranks {bad}"
        barrier(world)
        multi = {"gather_ms": gather_ms, "gather_bytes": int(full.numel() * 2), "gather_check": check,
                 "gather_check_how": "rank 0 recomputes every rank's shard (same seed) on its own GPU and "
                                     "compares it with that rank's slice of the all_gather output, bit for bit",
                 "scale_semantics": "per-tensor activation scales are taken over each rank's local batch "
                                    "(the reference quantises each linear's input as one tensor), so an "
                                    "N-GPU output differs from the 1-GPU one within FP8 rounding"}

    fp8pk = measure_fp8_peak(dev) if rank == 0 else None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from whisper_blaze_b200.encoder import EncoderConfig as _C
        ccfg = _C(layers=args.layers)
        info = cpu_reference_chunk(ccfg, cpu_layers(ccfg), args.cpu_budget)
        cpu = {"value": info["chunks_per_s"], "unit": "chunks/s", "cores": info["threads"], "kind": "port",
               "sample": f"1 chunk (1500 frames) x {info['layers_run']} of {ccfg.layers} layers timed "
                         f"({info['chunk_seconds'] / ccfg.layers * info['layers_run']:.1f} s), per-layer mean "
                         f"extrapolated to {ccfg.layers} layers; torch-CPU fp32 dequantise+matmul "
                         f"(oracle/encoder.py), fp32 SDPA"}

    if rank == 0:
        bf16x2, bf16x2_src = fp8_peak(sustained=True)
        peak = fp8pk["cublaslt_fp8_tflops_sustained"]
        peak_src = ("measured in this run: cuBLASLt FP8 E4M3 GEMM (torch._scaled_mm) 8192^3 back to back for "
                    "1 s under the power cap (the library-GEMM method of MEASURED_PEAKS.json's bf16 figure)")
        achieved = gemm_flops / (gemm_ms * 1e-3) / 1e12 if gemm_ms > 0 else None
        stack_mhz = clock_info.get("sm_mhz")
        pk_mhz = fp8pk.get("cublaslt_sustained_sm_mhz")
        frac_clk = (achieved / stack_mhz) / (peak / pk_mhz) if achieved and stack_mhz and pk_mhz else None
        value = TOTAL_CHUNKS / (ms * 1e-3)
        line = {
            "metric": "encoder chunks/s (32-layer FP8 Whisper-large-v3 encoder stack)",
            "value": value, "unit": "chunks/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "fp8 e4m3 (fp32 accumulate, fp16 activations, fp16 SDPA)", "data": "synthetic",
            "config": {"workload": "encoder_stack (config 5)", "global_batch": TOTAL_CHUNKS,
                       "seq_len": cfg.seq_len, "d_model": D, "heads": cfg.heads, "ffn": Fd, "layers": cfg.layers,
                       "parallelism": f"batch-sharded dp{world}, NCCL all_gather of outputs",
                       "slice_chunks": args.slice_chunks, "cuda_graph": bool(args.graph),
                       "l2": "inputs and every activation > 126 MB L2 (no flush needed)"},
            "e2e": {"value": TOTAL_CHUNKS / (e2e_ms * 1e-3), "unit": "chunks/s",
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h)},
            "roofline": {"bound": "tensor", "kernel": "wbk fp8_gemm_kernel (tcgen05 kind::f8f6f4)",
                         "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": (achieved / peak) if achieved else None, "peak_source": peak_src,
                         "frac_clock_normalised": frac_clk,
                         "frac_clock_normalised_how": "(achieved / the stack's median SM MHz) / (peak / the peak "
                                                      "run's median SM MHz)",
                         "fp8_peak_probe": fp8pk,
                         "frac_of_2x_bf16_sustained": (achieved / bf16x2) if achieved else None,
                         "bf16x2_source": bf16x2_src,
                         "frac_of_nominal_fp8_4500": (achieved / NOMINAL_FP8_TFLOPS) if achieved else None,
                         "gemm_launches_timed": n_gemm, "gemm_ms_per_step": gemm_ms / roofline_steps,
                         "gemm_share_of_step": (gemm_ms / roofline_steps) / ms_local,
                         "gemm_timing": ("CUDA events around each GEMM launch of " +
                                         (f"{roofline_steps} eager steps right after the timed graph replays"
                                          if args.graph else "the timed steps")),
                         "gemm_breakdown": breakdown,
                         "traffic": roofline_traffic("fp8_gemm_stack")},
            "gpu_launches": launches,
            "clocks": clock_info,
            "cpu_baseline": cpu,
        }
        if multi is not None:
            line["multi_gpu"] = multi
        print(json.dumps(line), flush=True)


# ------------------------------------------------------- secondary configs

def _graph_time(fn, steps: int, warmup: int, reps: int = 20) -> float:
    """Device milliseconds per call of fn: `reps` back-to-back calls captured in one
    CUDA graph (no host launch overhead between them), replayed `steps` times after
    `warmup` replays, timed with CUDA events."""
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            fn()
    for _ in range(max(1, warmup)):
        g.replay()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        g.replay()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / (steps * reps)


def run_gemm_configs(args, world, rank, local):
    """Configs 1-4: per-GEMM TFLOP/s (or GB/s for the memory-bound decoder step)."""
    from whisper_blaze_b200 import ops
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    wl = args.workload
    calls = set(args.calls.split(","))
    if wl == "fc1":
        shapes = [("fc1", 1500, 5120, 1280, "none")]
    elif wl == "layer":
        # as the stack runs them: fc1 with the bias + max-key epilogue (its GELU is applied by the
        # quantiser that feeds fc2, timed as fc1_gelu_quantise); fc1 with the GELU epilogue in the
        # GEMM is reported too (fc1_gelu_epilogue) but not counted in the total
        shapes = [("qkv", 24000, 3840, 1280, "none"), ("out_proj", 24000, 1280, 1280, "residual"),
                  ("fc1", 24000, 5120, 1280, "bias_maxkey"), ("fc2", 24000, 1280, 5120, "residual"),
                  ("fc1_gelu_epilogue", 24000, 5120, 1280, "gelu")]
    elif wl == "decoder":
        shapes = [(f"dec_n{n}", 64, n, 1280, "none") for n in (1280, 3840, 5120, 51866)]
    else:
        shapes = [("cross_kv", 48000, 2560, 1280, "none")]
    if args.shapes:
        keep = set(args.shapes.split(","))
        shapes = [sh for sh in shapes if sh[0] in keep]
        if not shapes:
            raise SystemExit(f"--shapes {args.shapes}: no such shape in workload {wl}")
    peak_t, src_t = fp8_peak(sustained=False)
    hbm = measured_peaks()["hbm_gbs"]
    results = {}
    tot_flops = tot_ms = tot_bytes = tot_dec_ms = 0.0
    cpu_on = rank == 0 and world == 1 and not args.no_cpu_baseline
    cpu_s = cpu_flops = cpu_bytes = 0.0
    if cpu_on:
        torch.set_num_threads(len(os.sched_getaffinity(0)))
    l2_bytes = 126e6
    for name, M, N, K, epi in shapes:
        x = torch.randn(M, K, generator=g, device=dev).half()
        w = (torch.randn(N, K, generator=g, device=dev) * 0.02).half()
        b = (torch.randn(N, generator=g, device=dev) * 0.02).half()
        res = torch.randn(M, N, generator=g, device=dev).half() if epi == "residual" else None
        key = ops.new_amax_ws(dev) if epi == "bias_maxkey" else None
        wq, sw = ops.quantise(w)
        # Timed calls rotate over enough copies of every operand that one pass moves
        # more than 1.5x the 126 MB L2, so no call reads another call's bytes from L2.
        per_call = 3 * M * K + N * K + 2 * M * N * (2 if res is not None else 1)
        copies = int(min(128, max(1, math.ceil(1.5 * l2_bytes / per_call))))
        sets = []
        for i in range(copies):
            st = types.SimpleNamespace(
                x=x if i == 0 else x.clone(), xq=torch.empty(M, K, dtype=torch.uint8, device=dev),
                sx=torch.empty(1, dtype=torch.float32, device=dev), ws=torch.empty(1, dtype=torch.int32, device=dev),
                wq=wq if i == 0 else wq.clone(), out=torch.empty(M, N, dtype=torch.float16, device=dev),
                res=None if res is None else (res if i == 0 else res.clone()))
            ops.quantise(st.x, q_out=st.xq, scale_out=st.sx, amax_ws=st.ws)
            sets.append(st)
        out = sets[0].out
        ctr = [0]

        def pick():
            st = sets[ctr[0] % copies]
            ctr[0] += 1
            return st

        def gemm_on(st):
            return ops.gemm_fp8(st.xq, st.sx, st.wq, sw, b, st.res, epi, out=st.out, out_amax=key)

        def quant_on(st):
            return ops.quantise(st.x, q_out=st.xq, scale_out=st.sx, amax_ws=st.ws)

        gemm = lambda: gemm_on(pick())  # noqa: E731
        quant = lambda: quant_on(pick())  # noqa: E731

        def both():
            st = pick()
            quant_on(st)
            gemm_on(st)

        def linear():  # the one-call public API (one cooperative kernel for M <= 128)
            st = pick()
            ops.linear_fp8(st.x, st.wq, sw, b, st.res, epi, out=st.out, out_amax=key, q_out=st.xq, scale_out=st.sx,
                           amax_ws=st.ws)

        reps = max(20, copies)
        timed = lambda f, what: _graph_time(f, args.steps, args.warmup, reps=reps) if what in calls else None  # noqa
        ms = timed(gemm, "gemm")
        qms = timed(quant, "quantise")
        bms = timed(both, "both")
        lms = timed(linear, "linear") if wl == "decoder" else None
        flops = 2.0 * M * N * K
        # decoder-step algorithmic bytes: 2MK (A fp16, quantised in-call) + NK (W fp8) + 2N (bias) + 2MN (out)
        dec_bytes = 2 * M * K + N * K + 2 * N + 2 * M * N
        results[name] = {"M": M, "N": N, "K": K, "epilogue": epi, "operand_copies": copies}
        if ms is not None:
            results[name].update({"gemm_ms": ms, "tflops": flops / ms / 1e9,
                                  "gemm_gbs_fp8_operands": (M * K + N * K + 2 * N + 2 * M * N) / ms / 1e6})
        if qms is not None:
            results[name].update({"quantise_A_ms": qms, "quantise_A_gbs": 3 * M * K / qms / 1e6})
        if bms is not None:
            results[name].update({"quantise_plus_gemm_ms": bms, "quantise_plus_gemm_gbs": dec_bytes / bms / 1e6})
        if lms is not None:
            results[name].update({"linear_fp8_ms": lms, "linear_fp8_gbs": dec_bytes / lms / 1e6})
        if epi == "bias_maxkey":
            # the GELU-quantise of the fc1 output that the stack runs next (HBM-bound: 2 B in, 1 B out)
            fq = torch.empty(M, N, dtype=torch.uint8, device=dev)
            fs = torch.empty(1, dtype=torch.float32, device=dev)
            gws = ops.new_amax_ws(dev)
            gq = lambda: ops.quantise_gelu(out, key, q_out=fq, scale_out=fs, amax_ws=gws)  # noqa: E731
            gms = _graph_time(gq, args.steps, args.warmup)
            results["fc1_gelu_quantise"] = {"M": M, "N": N, "ms": gms, "gbs": 3 * M * N / gms / 1e6}
        if name.endswith("_gelu_epilogue"):
            continue
        if cpu_on:  # the reference's CPU path on the same operands: one warm-up, one timed call
            xc, wc, sw_c = x.cpu(), wq.cpu(), float(sw.item())
            bc = b.cpu()
            rc = None if res is None else res.cpu()
            cpu_linear_seconds(xc, wc, sw_c, bc, rc, epi)
            t_cpu = cpu_linear_seconds(xc, wc, sw_c, bc, rc, epi)
            results[name]["cpu_ms"] = t_cpu * 1e3
            cpu_s += t_cpu
            cpu_flops += flops
            cpu_bytes += dec_bytes
        tot_flops += flops
        tot_ms += ms if ms is not None else float("nan")
        tot_bytes += dec_bytes
        tot_dec_ms += lms if lms is not None else (bms if bms is not None else float("nan"))
    if wl == "decoder":
        value = tot_bytes / tot_dec_ms / 1e6
        line = {"metric": "decoder-step FP8 linear HBM GB/s (quantise A in-call + GEMM, 4 shapes)", "value": value,
                "measured_call": "ops.linear_fp8 (fp16 A in; codes, scale and output out; one cooperative kernel "
                                 "that quantises A and runs the GEMM)",
                "unit": "GB/s",
                "roofline": {"bound": "hbm", "achieved": value, "peak": hbm, "unit": "GB/s", "frac": value / hbm,
                             "peak_source": "hbm_gbs of MEASURED_PEAKS.json"}}
    else:
        value = tot_flops / tot_ms / 1e9
        line = {"metric": "FP8 GEMM TFLOP/s", "value": value, "unit": "TFLOP/s",
                "roofline": {"bound": "tensor", "achieved": value, "peak": peak_t, "unit": "TFLOP/s",
                             "frac": value / peak_t, "peak_source": src_t,
                             "frac_of_nominal_fp8_4500": value / NOMINAL_FP8_TFLOPS}}
    if cpu_on and cpu_s > 0:
        line["cpu_baseline"] = {
            "value": (cpu_bytes / cpu_s / 1e9) if wl == "decoder" else (cpu_flops / cpu_s / 1e12),
            "unit": line["unit"], "cores": torch.get_num_threads(), "kind": "port",
            "sample": "one call per shape (after one warm-up) of the reference's CPU path on the same operands: "
                      "quantise the fp16 activation, fp32-dequantise both operands, fp32 matmul + bias + "
                      "epilogue, fp16 out (oracle/fp8.py quantise_torch, oracle/gemm.py)"}
    line.update({"n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                 "dtype": "fp8 e4m3", "data": "synthetic",
                 "timing": "CUDA graph of max(20, copies) back-to-back calls rotating over operand copies "
                           "(> 1.5x the 126 MB L2 per pass, so no call hits another's operands in L2), "
                           "device time per call",
                 "config": {"workload": wl, "shapes": results}})
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_attention(args, world, rank, local):
    """Encoder self-attention of the stack shape: `--chunks` x 20 heads x 1500 x 64 on the
    strided q/k/v views of a fused [T, 3840] QKV buffer, output into [T, 1280]; the tcgen05
    kernel against torch SDPA (cuDNN) on the same views. TFLOP/s = 4 B H S^2 Dh / t."""
    from whisper_blaze_b200 import ops
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    B, S, H, Dh = args.chunks, 1500, 20, 64
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    qkv = torch.randn(B * S, 3 * H * Dh, generator=g, device=dev).half()
    v5 = qkv.view(B, S, 3, H, Dh)
    q, k, v = (v5[:, :, i].transpose(1, 2) for i in range(3))
    out = torch.empty(B * S, H * Dh, dtype=torch.float16, device=dev)
    amax = ops.new_amax_ws(dev)
    ours = lambda: ops.attention(q, k, v, out=out.view(B, S, H, Dh).transpose(1, 2), out_amax=amax)  # noqa: E731
    sdpa = lambda: torch.nn.functional.scaled_dot_product_attention(q, k, v)  # noqa: E731
    flops = 4.0 * B * H * S * S * Dh
    ms = _graph_time(ours, args.steps, args.warmup, reps=4)
    ms_sdpa = _graph_time(sdpa, args.steps, args.warmup, reps=4)
    peak = measured_peaks().get("bf16_tflops")
    value = flops / ms / 1e9
    line = {"metric": "encoder self-attention TFLOP/s (fp16, head dim 64)", "value": value, "unit": "TFLOP/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "dtype": "fp16 (fp32 softmax and accumulate)", "data": "synthetic",
            "timing": "CUDA graph of 4 back-to-back calls, device time per call",
            "config": {"workload": "attention", "batch": B, "heads": H, "seq_len": S, "head_dim": Dh,
                       "layout": "strided views of a fused QKV buffer"},
            "ms_per_call": ms, "sdpa_ms_per_call": ms_sdpa, "sdpa_tflops": flops / ms_sdpa / 1e9,
            "roofline": {"bound": "tensor (exp throughput in practice)", "achieved": value, "peak": peak,
                         "unit": "TFLOP/s", "frac": value / peak if peak else None,
                         "peak_source": "bf16_tflops of MEASURED_PEAKS.json (dense fp16 = dense bf16 rate)"}}
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_norms(args, world, rank, local):
    """The norm ops of the op surface at the stack's shape (96000 x 1280 fp16, gamma = 1, beta = 0),
    HBM-bound: layernorm_fused, layernorm_fused_residual (normed + sum), rmsnorm_fused (with
    residual) and the fused LayerNorm -> FP8 pair. Algorithmic bytes per call (the LayerNorm rule):
    2 R D (1 + has_res + 1 + want_sum) + 2 D per parameter vector; LayerNorm -> FP8: 2 R D in +
    R D codes out. Each timing is a CUDA graph rotating over three inputs (each > the 126 MB L2)."""
    from whisper_blaze_b200 import ops
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    R, D = TOTAL_CHUNKS * 1500, 1280
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    xs = [torch.randn(R, D, generator=g, device=dev).half() for _ in range(3)]
    rs = [torch.randn(R, D, generator=g, device=dev).half() for _ in range(3)]
    gamma = torch.ones(D, dtype=torch.float16, device=dev)
    beta = torch.zeros(D, dtype=torch.float16, device=dev)
    out = torch.empty(R, D, dtype=torch.float16, device=dev)
    sm = torch.empty(R, D, dtype=torch.float16, device=dev)
    q = torch.empty(R, D, dtype=torch.uint8, device=dev)
    sc = torch.empty(1, dtype=torch.float32, device=dev)
    ws = ops.layernorm_quantise_ws(R, dev)
    am = ops.new_amax_ws(dev)
    ctr = [0]

    def nxt():
        ctr[0] += 1
        return ctr[0] % 3

    cases = [
        ("layernorm_fused", lambda: ops.layernorm(xs[nxt()], None, gamma, beta, out=out), 2 * R * D * 2 + 4 * D),
        ("layernorm_fused_residual", lambda: (lambda i: ops.layernorm(xs[i], rs[i], gamma, beta, want_sum=True,
                                                                       out=out, sum_out=sm))(nxt()),
         2 * R * D * 4 + 4 * D),
        ("rmsnorm_fused", lambda: (lambda i: ops.rmsnorm(xs[i], rs[i], gamma))(nxt()), 2 * R * D * 3 + 2 * D),
        ("layernorm_quantise", lambda: ops.layernorm_quantise(xs[nxt()], gamma, beta, q_out=q, scale_out=sc, ws=ws,
                                                               amax_ws=am), 3 * R * D + 4 * D),
    ]
    hbm = measured_peaks()["hbm_gbs"]
    results, tot_b, tot_ms = {}, 0.0, 0.0
    cpu_on = rank == 0 and world == 1 and not args.no_cpu_baseline
    cpu_b = cpu_s = 0.0
    if cpu_on:
        torch.set_num_threads(len(os.sched_getaffinity(0)))
        xc, rc_ = xs[0].cpu(), rs[0].cpu()
        gc, bc = gamma.cpu().float(), beta.cpu().float()
    for name, fn, nbytes in cases:
        ms = _graph_time(fn, args.steps, args.warmup, reps=30)
        results[name] = {"rows": R, "D": D, "us_per_call": ms * 1e3, "gbs": nbytes / ms / 1e6,
                         "frac_of_hbm": nbytes / ms / 1e6 / hbm}
        tot_b += nbytes
        tot_ms += ms
        if cpu_on:  # the reference's CPU path: torch fp32 layer_norm / rms norm of the same input
            t0 = time.perf_counter()
            xf = xc.float()
            if name == "rmsnorm_fused":
                h = xf + rc_.float()
                (h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + 1e-5) * gc).half()
            elif name == "layernorm_fused_residual":
                h = xf + rc_.float()
                torch.nn.functional.layer_norm(h, [D], gc, bc, 1e-5).half()
                h.half()
            else:
                torch.nn.functional.layer_norm(xf, [D], gc, bc, 1e-5).half()
            t = time.perf_counter() - t0
            results[name]["cpu_ms"] = t * 1e3
            cpu_b += nbytes
            cpu_s += t
    value = tot_b / tot_ms / 1e6
    line = {"metric": "norm ops HBM GB/s (layernorm_fused, _residual, rmsnorm_fused, LayerNorm->FP8; 96000 x 1280)",
            "value": value, "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "dtype": "fp16 (fp32 statistics)", "data": "synthetic",
            "timing": "CUDA graph of 30 calls rotating over 3 inputs (each > the 126 MB L2), device time per call",
            "roofline": {"bound": "hbm", "achieved": value, "peak": hbm, "unit": "GB/s", "frac": value / hbm,
                         "peak_source": "hbm_gbs of MEASURED_PEAKS.json"},
            "config": {"workload": "norms", "ops": results}}
    if cpu_on and cpu_s > 0:
        line["cpu_baseline"] = {"value": cpu_b / cpu_s / 1e9, "unit": "GB/s", "cores": torch.get_num_threads(),
                                "kind": "port", "sample": "one call per op of torch-CPU fp32 layer_norm / rms norm "
                                                          "on the same 96000 x 1280 input (fp16 out)"}
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_fp8peak(args, world, rank, local):
    """The measured dense FP8 ceiling alone (measure_fp8_peak): cuBLASLt FP8 GEMM and ours on 8192^3."""
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if rank != 0:
        return
    pk = measure_fp8_peak(dev, seconds=max(1.0, float(args.steps) / 10))
    v = pk["cublaslt_fp8_tflops_sustained"]
    line = {"metric": "dense FP8 E4M3 GEMM TFLOP/s (library GEMM, sustained)", "value": v, "unit": "TFLOP/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "dtype": "fp8 e4m3",
            "data": "synthetic", "config": {"workload": "fp8peak", "shape": pk["shape"]}, "probe": pk,
            "frac_of_nominal_fp8_4500": v / NOMINAL_FP8_TFLOPS}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["stack", "layer", "fc1", "decoder", "crossattn", "attention", "norms",
                                           "fp8peak"],
                    default="stack")
    ap.add_argument("--chunks", type=int, default=64, help="batch of the attention workload")
    ap.add_argument("--shapes", default="", help="comma-separated shape names to keep (gemm workloads; for profiling)")
    ap.add_argument("--calls", default="gemm,quantise,both,linear",
                    help="gemm workloads: which timings to run (gemm, quantise, both, linear; for profiling)")
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--cpu-budget", type=float, default=20.0)
    ap.add_argument("--ref-step-budget", type=float, default=8.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--graph", type=int, default=1, help="replay the stack from a CUDA graph (1) or launch eagerly (0)")
    ap.add_argument("--slice-chunks", type=int, default=int(os.environ.get("WBK_SLICE_CHUNKS", "0")),
                    help="chunks per pass through the stack (0 = the whole per-GPU batch at once)")
    args = ap.parse_args()
    world, rank, local = setup_dist()
    try:
        if args.impl == "reference":
            run_reference_arm(args, world, rank)
        elif args.workload == "stack":
            run_stack(args, world, rank, local)
        elif args.workload == "attention":
            run_attention(args, world, rank, local)
        elif args.workload == "norms":
            run_norms(args, world, rank, local)
        elif args.workload == "fp8peak":
            run_fp8peak(args, world, rank, local)
        else:
            run_gemm_configs(args, world, rank, local)
    finally:
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
