// Shared host + device helpers for libwbk (B200 / sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#include "wbk.h"

namespace wbk {

// ------------------------------------------------------------------ host side

// Records a printf-style message as this thread's last error and returns `code`.
int fail(int code, const char* fmt, ...);

// Maps a CUDA runtime error to WBK_ERR_CUDA (with message) or WBK_OK.
int cuda_check(cudaError_t e, const char* what);

// Number of SMs of the current device (cached per device).
int sm_count();

// Current device ordinal, or -1 on failure.
int current_device();

inline bool aligned(const void* p, size_t a) {
  return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
}

// ---------------------------------------------------------------- device side

// |x| of two packed fp16 values with NaN lanes forced to 0 (so a max over
// them ignores NaN, like fmaxf does). Infinity stays 0x7C00.
__device__ __forceinline__ uint32_t abs2_nonan(uint32_t w) {
  const uint32_t a = w & 0x7FFF7FFFu;
  const uint32_t nan_mask = __vcmpgtu2(a, 0x7C007C00u);  // 0xFFFF per NaN lane
  return a & ~nan_mask;
}

// fp16 bit pattern -> float (exact).
__device__ __forceinline__ float half_bits_to_float(uint32_t bits) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(bits & 0xFFFFu)));
}

// max over a warp of an unsigned value.
__device__ __forceinline__ uint32_t warp_max_u32(uint32_t v) {
  return __reduce_max_sync(0xFFFFFFFFu, v);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

// Streaming 16-byte global load (read once, keep L1 clean).
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

}  // namespace wbk
