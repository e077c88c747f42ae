"""B200-native FP8 quantised-matmul path of whisper-blaze.

Host-side package over libwbk.so (hand-written sm_100a kernels, C ABI in
include/wbk.h):
  ops        tensor wrappers: quantise / dequantise / layernorm / rmsnorm / gemm_fp8
  precision  PrecisionConfig mirror, with a real `fp8_e4m3` preset
  modules    BlazeLinear (FP8 GEMM) and BlazeLayerNorm
  encoder    Whisper-large-v3-shaped FP8 encoder stack
  sharding   batch partitioning across GPUs + one NCCL gather
The drop-in op module is `whisper_blaze_kernels` (same directory level).
"""
from . import ops, precision  # noqa: F401
from ._lib import LIB_PATH, WbkError  # noqa: F401

__version__ = "0.1.0"
