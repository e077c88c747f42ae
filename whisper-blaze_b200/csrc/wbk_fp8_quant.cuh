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

// Two fp32 products a.x * s, a.y * s in one instruction (f2_mul).
__device__ __forceinline__ float2 mul2_rn(float2 a, float s) { return f2_mul(a, make_float2(s, s)); }

// The codes of q8x4 for any finite inv > 0 (inv is 0 only when the amax is
// infinite; callers take q8x4 then), in fewer instructions:
//  * a NaN lane becomes -65504 first (max.f16x2 returns the operand that is not
//    NaN). The amax is an fp16 value, so 65504 >= amax and 65504 * inv is at
//    least max_fp8 up to the rounding of the scale: the saturating
//    round-to-nearest conversion gives -max_fp8, as the clamp gave for NaN (the
//    nearest other codes, 416 and 49152, are far away);
//  * every other product converts as after the clamp to [-max_fp8, max_fp8],
//    because .satfinite saturates to +-max_fp8 exactly where the clamp would
//    (infinities included);
//  * the two fp32 products of a pair are one mul.rn.f32x2.
template <int kFmt>
__device__ __forceinline__ uint32_t q8x4_fin(uint32_t h01, uint32_t h23, float inv) {
  constexpr uint32_t kNegMax2 = 0xFBFFFBFFu;  // two fp16 -65504
  uint32_t a, b;
  asm("max.f16x2 %0, %1, %2;" : "=r"(a) : "r"(h01), "r"(kNegMax2));
  asm("max.f16x2 %0, %1, %2;" : "=r"(b) : "r"(h23), "r"(kNegMax2));
  const float2 f01 = mul2_rn(__half22float2(*reinterpret_cast<const __half2*>(&a)), inv);
  const float2 f23 = mul2_rn(__half22float2(*reinterpret_cast<const __half2*>(&b)), inv);
  constexpr __nv_fp8_interpretation_t it = kFmt == WBK_FMT_E4M3 ? __NV_E4M3 : __NV_E5M2;
  return static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(f01, __NV_SATFINITE, it)) |
         (static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(f23, __NV_SATFINITE, it)) << 16);
}

// Eight fp16 values (one 16-byte vector) -> eight fp8 codes; kFin selects
// q8x4_fin (valid for finite inv > 0) over q8x4.
template <int kFmt, bool kFin>
__device__ __forceinline__ uint2 q8x8(const uint4& v, float inv, float mx) {
  if constexpr (kFin) return make_uint2(q8x4_fin<kFmt>(v.x, v.y, inv), q8x4_fin<kFmt>(v.z, v.w, inv));
  else return make_uint2(q8x4<kFmt>(v.x, v.y, inv, mx), q8x4<kFmt>(v.z, v.w, inv, mx));
}

// Running max of |x| over two packed fp16 values, NaN ignored: max.f16x2
// returns the operand that is not NaN, and an accumulator started at 0 never
// holds a NaN. Both halves hold the fp16 bits of values >= 0, whose unsigned
// order is their numeric order, so the lanes equal the unsigned max of
// abs2_nonan's lanes.
__device__ __forceinline__ uint32_t hmax_abs2(uint32_t acc, uint32_t w) {
  uint32_t r;
  asm("max.f16x2 %0, %1, %2;" : "=r"(r) : "r"(acc), "r"(w & 0x7FFF7FFFu));
  return r;
}

// Running max of |x| over one 16-byte vector of fp16 into a packed accumulator.
__device__ __forceinline__ uint32_t absmax8_acc(uint32_t acc, const uint4& v) {
  return hmax_abs2(hmax_abs2(hmax_abs2(hmax_abs2(acc, v.x), v.y), v.z), v.w);
}

// The packed accumulator's two lanes -> one fp16 bit pattern.
__device__ __forceinline__ uint32_t absmax_lanes(uint32_t acc) { return max(acc & 0xFFFFu, acc >> 16); }

// max |x| over eight fp16 values (one 16-byte vector) as fp16 bits, NaN ignored.
__device__ __forceinline__ uint32_t absmax8_bits(const uint4& v) { return absmax_lanes(absmax8_acc(0u, v)); }

}  // namespace wbk
