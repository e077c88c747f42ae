"""CPU oracle for the FP8 quantised-matmul path of whisper-blaze.

TEST INFRASTRUCTURE ONLY. Nothing in the product (the `whisper-blaze_b200`
package or libwbk.so) imports, calls or links this package; only `tests/`,
`__graft_entry__.smoke()` and the `cpu_baseline` / `--impl reference` legs of
`bench.py` use it, and only as the checker or as the timed CPU reference path.

It restates, in numpy and torch-CPU fp32, what the reference computes:

* fp8.py    — per-tensor amax/scale, E4M3/E5M2 quantise and dequantise
              (csrc/kernels/fp8_quantize.cu), with an independent table-based
              round-to-nearest-even fp8 encoder;
* gemm.py   — FP8 linear = fp32 matmul of the dequantised operands plus the
              bias / GELU / residual epilogues (whisper_blaze/model.py:80-109,
              csrc/kernels/gemm_hopper.cu:251-268);
* norm.py   — fused residual + LayerNorm / RMSNorm
              (csrc/kernels/layernorm_fused.cu);
* encoder.py — the Whisper encoder layer with FP8 linears (HF
              WhisperEncoderLayer structure) and the CPU timing harness.

Pinning: the reference ships no golden vectors for this path. The oracle is
pinned (a) by the reference's own test assertions (tests/test_kernels.py,
tests/test_precision.py), restated in tests/test_oracle_*.py, and (b) by golden
fixtures produced by the reference's own CUDA kernels (fp8_quantize.cu and
layernorm_fused.cu built unmodified from the reference sources into
oracle/_ref/ by oracle/build_ref.py and run on a B200 by
tests/golden/make_golden.py).
"""
