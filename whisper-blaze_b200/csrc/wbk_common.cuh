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

// Reads (and optionally clears) the device error word of the attention unit.
int attn_read_device_error(uint32_t* v, bool clear);

// Wall-clock limit of the bounded device waits set by wbk_set_wait_timeout_ns
// (0 = not set: the WBK_WAIT_TIMEOUT_MS / 4 s default applies).
uint64_t wait_timeout_override_ns();

inline bool aligned(const void* p, size_t a) {
  return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
}

// ---------------------------------------------------------------- device side

// Packed fp32 pairs (sm_100 add / mul / fma .rn.f32x2, one instruction for two
// lanes): each lane is rounded exactly as the scalar operation would round it.
__device__ __forceinline__ float2 f2_add(float2 a, float2 b) {
  float2 r;
  asm("{\n\t.reg .b64 a, b, d;\n\tmov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\t"
      "add.rn.f32x2 d, a, b;\n\tmov.b64 {%0, %1}, d;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}
__device__ __forceinline__ float2 f2_mul(float2 a, float2 b) {
  float2 r;
  asm("{\n\t.reg .b64 a, b, d;\n\tmov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\t"
      "mul.rn.f32x2 d, a, b;\n\tmov.b64 {%0, %1}, d;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}
__device__ __forceinline__ float2 f2_fma(float2 a, float2 b, float2 c) {
  float2 r;
  asm("{\n\t.reg .b64 a, b, c, d;\n\tmov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\tmov.b64 c, {%6, %7};\n\t"
      "fma.rn.f32x2 d, a, b, c;\n\tmov.b64 {%0, %1}, d;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return r;
}

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

// erf(z) for z >= 0 by Abramowitz & Stegun, Handbook of Mathematical Functions,
// formula 7.1.26: erf(z) = 1 - (a1 t + a2 t^2 + a3 t^3 + a4 t^4 + a5 t^5) e^{-z^2},
// t = 1 / (1 + p z), |error| <= 1.5e-7 — far below the fp16 resolution of a
// GELU output — for about a third of the FMA-pipe work of erff.
__device__ __forceinline__ float erf_nonneg_as7126(float z) {
  const float t = __fdividef(1.0f, fmaf(0.3275911f, z, 1.0f));
  float poly = fmaf(t, 1.061405429f, -1.453152027f);
  poly = fmaf(t, poly, 1.421413741f);
  poly = fmaf(t, poly, -0.284496736f);
  poly = fmaf(t, poly, 0.254829592f);
  poly *= t;
  const float e = exp2f(-z * z * 1.4426950408889634f);  // e^{-z^2}
  return fmaf(-poly, e, 1.0f);
}

// Exact-erf GELU (HF activation "gelu"): 0.5 v (1 + erf(v / sqrt 2)).
__device__ __forceinline__ float gelu_erf(float v) {
  const float z = fabsf(v) * 0.70710678118654752440f;
  const float er = copysignf(erf_nonneg_as7126(z), v);
  return 0.5f * v * (1.0f + er);
}

// Order-preserving key of an fp16 bit pattern, so an unsigned atomicMax finds
// the largest (signed) value; key 0 means "no value".
__device__ __forceinline__ uint32_t f16_order_key(uint32_t h) {
  h &= 0xFFFFu;
  return (h & 0x8000u) ? (~h & 0xFFFFu) : (h | 0x8000u);
}
__device__ __forceinline__ uint32_t f16_from_order_key(uint32_t k) {
  return (k & 0x8000u) ? (k & 0x7FFFu) : (~k & 0xFFFFu);
}

// Programmatic dependent launch. A kernel launched with the programmatic
// stream-serialization attribute may start while the previous kernel in the
// stream still runs; it calls griddep_wait() before touching anything that
// kernel writes (the wait returns once the previous grid has completed and its
// memory is visible). Producers call griddep_launch_dependents() to let such a
// dependant start early. Both are no-ops for ordinary launches.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Streaming 16-byte global load (read once, keep L1 clean).
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

// L2 eviction-priority policies (createpolicy) and a streaming 16-byte load that
// carries one: evict_last keeps lines a later pass re-reads, evict_first marks
// a last use.
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ uint4 ld_stream16_hint(const void* p, uint64_t pol) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p), "l"(pol));
  return r;
}

}  // namespace wbk
