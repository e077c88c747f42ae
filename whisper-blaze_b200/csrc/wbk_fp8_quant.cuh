// Per-tensor FP8 quantisation arithmetic shared by the quantiser kernels and
// the GEMM that quantises its own activations, so both produce the same codes
// and scales bit for bit whatever the translation unit's math flags.
#pragma once

#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#include "wbk_common.cuh"

namespace wbk {

// Largest finite value of the format (E4M3: 448, E5M2: 57344).
__host__ __device__ constexpr float fmt_max(int fmt) { return fmt == WBK_FMT_E4M3 ? 448.0f : 57344.0f; }

// The reference's scale rule: scale = amax / max_fp8, replaced by 1.0 unless
// it is > 0 (fp8_quantize.cu:72 and :218); inv_scale = 1/scale rounded to
// nearest (host IEEE division at fp8_quantize.cu:224; __frcp_rn is the
// correctly rounded reciprocal, so the two agree for every scale).
// The reference kernel is built with fast math, where amax / max_fp8 is the
// approximate quotient; __fdividef names that quotient explicitly (checked on
// B200 against the reference's scale for every positive fp16 amax, both
// formats), so the result does not depend on this unit's own flags.
__device__ __forceinline__ void scale_from_amax(uint32_t amax_bits, float max_fp8, float& scale, float& inv) {
  const float amax = half_bits_to_float(amax_bits);
  float s = __fdividef(amax, max_fp8);
  s = (s > 0.0f) ? s : 1.0f;
  scale = s;
  inv = __frcp_rn(s);
}

// Two values -> two fp8 codes (low byte first): x * inv clamped to
// [-max_fp8, max_fp8] (NaN becomes -max_fp8 through fmaxf), then the
// saturating round-to-nearest-even conversion.
template <int kFmt>
__device__ __forceinline__ uint32_t q8x2(float a, float b, float inv, float mx) {
  float2 f;
  f.x = fminf(fmaxf(a * inv, -mx), mx);
  f.y = fminf(fmaxf(b * inv, -mx), mx);
  return __nv_cvt_float2_to_fp8x2(f, __NV_SATFINITE, kFmt == WBK_FMT_E4M3 ? __NV_E4M3 : __NV_E5M2);
}

// Four packed fp16 values (two half2 words) -> four fp8 codes.
template <int kFmt>
__device__ __forceinline__ uint32_t q8x4(uint32_t h01, uint32_t h23, float inv, float mx) {
  const float2 f01 = __half22float2(*reinterpret_cast<const __half2*>(&h01));
  const float2 f23 = __half22float2(*reinterpret_cast<const __half2*>(&h23));
  return q8x2<kFmt>(f01.x, f01.y, inv, mx) | (q8x2<kFmt>(f23.x, f23.y, inv, mx) << 16);
}

// max |x| over eight fp16 values (one 16-byte vector) as fp16 bits, NaN ignored.
__device__ __forceinline__ uint32_t absmax8_bits(const uint4& v) {
  const uint32_t m = __vmaxu2(__vmaxu2(abs2_nonan(v.x), abs2_nonan(v.y)), __vmaxu2(abs2_nonan(v.z), abs2_nonan(v.w)));
  return max(m & 0xFFFFu, m >> 16);
}

}  // namespace wbk
