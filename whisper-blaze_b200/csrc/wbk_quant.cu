// Per-tensor FP8 (E4M3 / E5M2) amax, quantise and dequantise kernels for B200.
//
// The scale rule and the per-element conversion live in wbk_fp8_quant.cuh,
// shared with the GEMM that quantises its own activations. The reference
// builds its quantiser with fast math (setup.py:41-54), so its
// compute_scale_kernel (csrc/kernels/fp8_quantize.cu:72) divides with the
// approximate quotient; the shared rule names that quotient (__fdividef).
// This unit keeps --use_fast_math for its other arithmetic, all of which is
// exact in either mode: fp16->fp32 conversion, one fp32 multiply per element
// (no fp32 denormals arise from fp16 inputs and these scales), fminf/fmaxf
// and the hardware round-to-nearest-even, saturate-to-finite fp8 conversion.
//
// Layout in HBM: the input is a flat fp16 array (any shape, contiguous); the
// output is a flat uint8 array of the same element count. Each thread moves
// 8 elements per step: one 16-byte load in, one 8-byte store out.
#include <cuda.h>
#include <mutex>
#include <vector>

#include "wbk_common.cuh"
#include "wbk_fp8_quant.cuh"

namespace wbk {
namespace {

constexpr int kThreads = 256;


// -------------------------------------------------------------------- amax

// Grid-stride max(|x|) over n fp16 values, NaN ignored, as a packed fp16 max
// (hmax_abs2). One atomicMax per CTA into *amax_bits.
template <bool kVec>
__global__ void __launch_bounds__(kThreads)
amax_f16_kernel(const __half* __restrict__ x, int64_t n, uint32_t* __restrict__ amax_bits) {
  uint32_t m = 0;  // two packed running maxima
  const uint64_t keep = l2_policy_evict_last();  // the quantise pass re-reads these lines
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  int64_t done = 0;
  if (kVec) {
    const int64_t nvec = n >> 3;
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    constexpr int kU = 8;  // 16-byte loads in flight per thread
    int64_t i = tid;
    for (; i + (kU - 1) * stride < nvec; i += kU * stride) {
      uint4 v[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) v[u] = ld_stream16_hint(xv + i + u * stride, keep);
#pragma unroll
      for (int u = 0; u < kU; ++u) m = absmax8_acc(m, v[u]);
    }
    for (; i < nvec; i += stride) m = absmax8_acc(m, ld_stream16_hint(xv + i, keep));
    done = nvec << 3;
  }
  const unsigned short* xs = reinterpret_cast<const unsigned short*>(x);
  for (int64_t i = done + tid; i < n; i += stride) m = hmax_abs2(m, xs[i]);

  uint32_t mm = absmax_lanes(m);
  mm = warp_max_u32(mm);
  __shared__ uint32_t red[kThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = mm;
  __syncthreads();
  if (warp == 0) {
    mm = lane < kThreads / 32 ? red[lane] : 0u;
    mm = warp_max_u32(mm);
    if (lane == 0 && mm != 0u) atomicMax(amax_bits, mm);
  }
}

// ---------------------------------------------------------------- quantise

// Codes of the 16-byte vectors [0, nvec) in grid-stride rounds from the LAST to
// the first: the amax pass that ran just before read the tensor front to back,
// so its most recent lines -- the ones still in L2 -- are read first here. Only
// the order changes. kFin: inv is finite and > 0 (q8x4_fin's condition).
template <int kFmt, bool kFin>
__device__ __forceinline__ void quantise_vectors_back(const uint4* __restrict__ xv, uint2* __restrict__ qv, int64_t nvec,
                                                      int64_t tid, int64_t stride, float inv, float max_fp8) {
  const int64_t rounds = (nvec + stride - 1) / stride;
  const uint64_t drop = l2_policy_evict_first();  // last use of the input
  int64_t r = rounds - 1;
  constexpr int kU = 4;  // rounds per step: 16-byte loads in flight per thread
  for (; r >= kU - 1; r -= kU) {  // rounds r .. r - kU + 1 (all but round r are full)
    uint4 v[kU];
    const int64_t i0 = r * stride + tid;
    const bool has0 = i0 < nvec;
    v[0] = has0 ? ld_stream16_hint(xv + i0, drop) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int u = 1; u < kU; ++u) v[u] = ld_stream16_hint(xv + i0 - u * stride, drop);
    if (has0) qv[i0] = q8x8<kFmt, kFin>(v[0], inv, max_fp8);
#pragma unroll
    for (int u = 1; u < kU; ++u) qv[i0 - u * stride] = q8x8<kFmt, kFin>(v[u], inv, max_fp8);
  }
  for (; r >= 0; --r) {  // the last rounds one at a time (round r may be partial only when it is the first)
    const int64_t i = r * stride + tid;
    if (i < nvec) qv[i] = q8x8<kFmt, kFin>(ld_stream16_hint(xv + i, drop), inv, max_fp8);
  }
}

template <int kFmt, bool kVec>
__global__ void __launch_bounds__(kThreads)
quantise_f16_kernel(const __half* __restrict__ x, int64_t n, const uint32_t* __restrict__ amax_bits,
                    float max_fp8, uint8_t* __restrict__ q, float* __restrict__ scale_out) {
  griddep_launch_dependents();  // a following GEMM may run its prologue meanwhile
  float scale, inv;
  scale_from_amax(*amax_bits, max_fp8, scale, inv);
  if (scale_out != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *scale_out = scale;

  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  int64_t done = 0;
  if (kVec) {
    const int64_t nvec = n >> 3;
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    uint2* qv = reinterpret_cast<uint2*>(q);
    if (inv != 0.0f) quantise_vectors_back<kFmt, true>(xv, qv, nvec, tid, stride, inv, max_fp8);
    else quantise_vectors_back<kFmt, false>(xv, qv, nvec, tid, stride, inv, max_fp8);  // an infinite amax
    done = nvec << 3;
  }
  for (int64_t i = done + tid; i < n; i += stride) {
    const float f = __half2float(x[i]);
    q[i] = static_cast<uint8_t>(q8x2<kFmt>(f, 0.0f, inv, max_fp8) & 0xFFu);
  }
}

// One thread: scale_inv[0] = scale, scale_inv[1] = 1/scale, from an amax (the
// same rule and the same compiled division as the quantise kernels above).
__global__ void scale_from_amax_kernel(const uint32_t* __restrict__ amax_bits, float max_fp8,
                                       float* __restrict__ scale_inv) {
  float scale, inv;
  scale_from_amax(*amax_bits, max_fp8, scale, inv);
  scale_inv[0] = scale;
  scale_inv[1] = inv;
}

// ------------------------------------------------------- GELU + quantise
//
// The FFN activation of the encoder is quantised right after the GELU. Here
// the GELU runs inside the quantiser pass (this pass reads the fc1 output
// anyway), on the fp16 fc1 output, rounded to fp16 like the stored GELU
// output of the reference path: g = fp16(gelu(float(y))).
//
// The per-tensor amax of g normally needs its own pass over y. It does not
// here: GELU is increasing for y >= -0.7518 and |gelu(y)| <= 0.16997 below
// that, and rounding to fp16 is monotone, so when g(y_max) >= 0.171 the amax of
// g is exactly g(y_max), where y_max is the largest fc1 output — which the
// GEMM epilogue already tracks (WBK_EPI_BIAS_MAXKEY). Otherwise a full pass
// computes max |g| element by element.

constexpr float kGeluNegativeMaxAbs = 0.171f;  // > max over y < 0 of |fp16(gelu(y))| (0.1700)

__device__ __forceinline__ uint32_t gelu_f16_bits(uint32_t h) {
  return __half_as_ushort(__float2half_rn(gelu_erf(half_bits_to_float(h))));
}

template <bool kVec>
__global__ void __launch_bounds__(kThreads)
gelu_amax_kernel(const __half* __restrict__ y, int64_t n, const uint32_t* __restrict__ ymax_key,
                 uint32_t* __restrict__ amax_bits) {
  if (ymax_key != nullptr) {
    const uint32_t key = *ymax_key;
    if (key != 0u) {
      const uint32_t g = gelu_f16_bits(f16_from_order_key(key));
      const float gf = half_bits_to_float(g);
      if (gf >= kGeluNegativeMaxAbs) {  // false for NaN
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicMax(amax_bits, g & 0x7FFFu);
        return;  // uniform across the grid: every CTA reads the same key
      }
    }
  }
  uint32_t m = 0;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  int64_t done = 0;
  if (kVec) {
    const int64_t nvec = n >> 3;
    const uint4* yv = reinterpret_cast<const uint4*>(y);
    for (int64_t i = tid; i < nvec; i += stride) {
      const uint4 v = ld_stream16(yv + i);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t g = gelu_f16_bits(w[k]) | (gelu_f16_bits(w[k] >> 16) << 16);
        m = __vmaxu2(m, abs2_nonan(g));
      }
    }
    done = nvec << 3;
  }
  const unsigned short* ys = reinterpret_cast<const unsigned short*>(y);
  for (int64_t i = done + tid; i < n; i += stride) m = __vmaxu2(m, abs2_nonan(gelu_f16_bits(ys[i])));
  uint32_t mm = warp_max_u32(max(m & 0xFFFFu, m >> 16));
  __shared__ uint32_t red[kThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = mm;
  __syncthreads();
  if (warp == 0) {
    mm = warp_max_u32(lane < kThreads / 32 ? red[lane] : 0u);
    if (lane == 0 && mm != 0u) atomicMax(amax_bits, mm);
  }
}

template <int kFmt>
__device__ __forceinline__ uint32_t gelu_q8x4(uint32_t h01, uint32_t h23, float inv, float mx) {
  const uint32_t g01 = gelu_f16_bits(h01) | (gelu_f16_bits(h01 >> 16) << 16);
  const uint32_t g23 = gelu_f16_bits(h23) | (gelu_f16_bits(h23 >> 16) << 16);
  return q8x4<kFmt>(g01, g23, inv, mx);
}

// The GELU output g = fp16(gelu(float(y))) depends only on the 16 bits of y,
// so each CTA first evaluates it once for all 65536 fp16 bit patterns into a
// 128 KB shared-memory table (with the same device function, so the result is
// bit-identical to evaluating it per element) and then needs one table lookup
// per element: the pass becomes HBM-bound instead of FMA-bound.
constexpr int kGeluThreads = 1024;
constexpr size_t kGeluTableBytes = 65536 * sizeof(uint16_t);

// The table never changes, so CTA 0 of the first launch that builds it also
// publishes it here (one copy per device, 128 KB, held until the library is
// unloaded); CTAs that find it published copy it from L2 instead of evaluating
// erf 65536 times.
__device__ __align__(16) uint16_t g_gelu_table[65536];
__device__ uint32_t g_gelu_table_ready;

// Fills the shared-memory table of this CTA (all threads call it).
__device__ __forceinline__ void load_gelu_table(uint16_t* table) {
  __shared__ uint32_t ready;
  if (threadIdx.x == 0) asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(ready) : "l"(&g_gelu_table_ready) : "memory");
  __syncthreads();
  uint4* t4 = reinterpret_cast<uint4*>(table);
  uint4* g4 = reinterpret_cast<uint4*>(g_gelu_table);
  if (ready) {
    for (int i = threadIdx.x; i < 65536 / 8; i += blockDim.x) t4[i] = __ldcg(g4 + i);
    return;
  }
  for (uint32_t h = threadIdx.x; h < 65536u; h += blockDim.x) table[h] = static_cast<uint16_t>(gelu_f16_bits(h));
  if (blockIdx.x != 0) return;
  __syncthreads();
  for (int i = threadIdx.x; i < 65536 / 8; i += blockDim.x) __stcg(g4 + i, t4[i]);
  __syncthreads();
  if (threadIdx.x == 0) asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(&g_gelu_table_ready), "r"(1u) : "memory");
}

__device__ __forceinline__ uint32_t gelu_lookup2(const uint16_t* table, uint32_t h2) {
  return static_cast<uint32_t>(table[h2 & 0xFFFFu]) | (static_cast<uint32_t>(table[h2 >> 16]) << 16);
}

template <int kFmt, bool kFin>
__device__ __forceinline__ uint2 gelu_q8x8(const uint16_t* table, const uint4& v, float inv, float mx) {
  const uint4 g = make_uint4(gelu_lookup2(table, v.x), gelu_lookup2(table, v.y), gelu_lookup2(table, v.z),
                             gelu_lookup2(table, v.w));
  return q8x8<kFmt, kFin>(g, inv, mx);
}

// Codes of the 16-byte vectors [0, nvec) of y's GELU (grid-stride, four per
// thread per step). kFin: inv is finite and > 0 (q8x4_fin's condition).
template <int kFmt, bool kFin>
__device__ __forceinline__ void gelu_quantise_vectors(const uint16_t* table, const uint4* __restrict__ yv,
                                                      uint2* __restrict__ qv, int64_t nvec, int64_t tid,
                                                      int64_t stride, float inv, float mx) {
  constexpr int kU = 8;  // 16-byte loads in flight per thread
  int64_t i = tid;
  for (; i + (kU - 1) * stride < nvec; i += kU * stride) {
    uint4 v[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) v[u] = ld_stream16(yv + i + u * stride);
#pragma unroll
    for (int u = 0; u < kU; ++u) qv[i + u * stride] = gelu_q8x8<kFmt, kFin>(table, v[u], inv, mx);
  }
  for (; i < nvec; i += stride) qv[i] = gelu_q8x8<kFmt, kFin>(table, ld_stream16(yv + i), inv, mx);
}

template <int kFmt, bool kVec>
__global__ void __launch_bounds__(kGeluThreads, 1)
quantise_gelu_kernel(const __half* __restrict__ y, int64_t n, const uint32_t* __restrict__ amax_bits,
                     float max_fp8, uint8_t* __restrict__ q, float* __restrict__ scale_out) {
  griddep_launch_dependents();  // a following GEMM may run its prologue meanwhile
  extern __shared__ uint16_t gelu_table[];
  load_gelu_table(gelu_table);
  float scale, inv;
  scale_from_amax(*amax_bits, max_fp8, scale, inv);
  if (scale_out != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *scale_out = scale;
  __syncthreads();
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  int64_t done = 0;
  if (kVec) {
    const int64_t nvec = n >> 3;
    const uint4* yv = reinterpret_cast<const uint4*>(y);
    uint2* qv = reinterpret_cast<uint2*>(q);
    if (inv != 0.0f) gelu_quantise_vectors<kFmt, true>(gelu_table, yv, qv, nvec, tid, stride, inv, max_fp8);
    else gelu_quantise_vectors<kFmt, false>(gelu_table, yv, qv, nvec, tid, stride, inv, max_fp8);  // infinite amax
    done = nvec << 3;
  }
  const unsigned short* ys = reinterpret_cast<const unsigned short*>(y);
  for (int64_t i = done + tid; i < n; i += stride) {
    const float g = half_bits_to_float(gelu_table[ys[i]]);
    q[i] = static_cast<uint8_t>(q8x2<kFmt>(g, 0.0f, inv, max_fp8) & 0xFFu);
  }
}

template <int kFmt, bool kVec>
int launch_quantise_gelu(const __half* y, int64_t n, const uint32_t* amax, float mx, uint8_t* q, float* scale_out,
                         cudaStream_t s) {
  static std::mutex mu;
  static std::vector<char> configured;
  const int dev = current_device();
  if (dev < 0) return fail(WBK_ERR_CUDA, "wbk_quantise_gelu_f16: no current CUDA device");
  {
    std::lock_guard<std::mutex> lock(mu);
    if (static_cast<int>(configured.size()) <= dev) configured.resize(dev + 1, 0);
    if (!configured[dev]) {
      if (int e = cuda_check(cudaFuncSetAttribute(quantise_gelu_kernel<kFmt, kVec>,
                                                  cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  static_cast<int>(kGeluTableBytes)),
                             "wbk_quantise_gelu_f16: cudaFuncSetAttribute"))
        return e;
      configured[dev] = 1;
    }
  }
  const int sms = sm_count() > 0 ? sm_count() : 148;
  const int64_t want = ((kVec ? (n + 7) / 8 : n) + kGeluThreads - 1) / kGeluThreads;
  const int grid = static_cast<int>(want < 1 ? 1 : (want < sms ? want : sms));
  quantise_gelu_kernel<kFmt, kVec><<<grid, kGeluThreads, kGeluTableBytes, s>>>(y, n, amax, mx, q, scale_out);
  return cuda_check(cudaGetLastError(), "wbk_quantise_gelu_f16 launch");
}

// ------------------------------------------------- small-tensor quantise
//
// For small tensors (the decoder step's 64 x 1280 activation) three launches
// (memset, amax, quantise) cost more than the data movement. One CTA does all
// of it: amax, the scale, then the quantise pass over the (now L1/L2 resident)
// input — the same scale rule and element rule as the two-kernel path.
constexpr int kSmallThreads = 1024;
constexpr int64_t kSmallQuantMax = 262144;  // elements (512 KB of fp16)

template <int kFmt, bool kVec>
__global__ void __launch_bounds__(kSmallThreads, 1)
quantise_small_kernel(const __half* __restrict__ x, int64_t n, float max_fp8, uint8_t* __restrict__ q,
                      float* __restrict__ scale_out, uint32_t* __restrict__ amax_out) {
  griddep_launch_dependents();  // a following GEMM may run its prologue meanwhile
  __shared__ uint32_t red[kSmallThreads / 32];
  __shared__ float sc[2];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t nvec = kVec ? (n >> 3) : 0;
  uint32_t m = 0;
  const uint4* xv = reinterpret_cast<const uint4*>(x);
  for (int64_t i = threadIdx.x; i < nvec; i += kSmallThreads) {
    const uint4 v = xv[i];
    m = __vmaxu2(m, __vmaxu2(__vmaxu2(abs2_nonan(v.x), abs2_nonan(v.y)), __vmaxu2(abs2_nonan(v.z), abs2_nonan(v.w))));
  }
  const unsigned short* xs = reinterpret_cast<const unsigned short*>(x);
  for (int64_t i = (nvec << 3) + threadIdx.x; i < n; i += kSmallThreads) m = __vmaxu2(m, abs2_nonan(xs[i]));
  uint32_t mm = warp_max_u32(max(m & 0xFFFFu, m >> 16));
  if (lane == 0) red[warp] = mm;
  __syncthreads();
  if (warp == 0) {
    mm = warp_max_u32(red[lane]);
    if (lane == 0) {
      float scale, inv;
      scale_from_amax(mm, max_fp8, scale, inv);
      sc[0] = scale;
      sc[1] = inv;
      if (scale_out != nullptr) *scale_out = scale;
      if (amax_out != nullptr) *amax_out = mm;
    }
  }
  __syncthreads();
  const float inv = sc[1];
  uint2* qv = reinterpret_cast<uint2*>(q);
  for (int64_t i = threadIdx.x; i < nvec; i += kSmallThreads) {
    const uint4 v = xv[i];
    qv[i] = make_uint2(q8x4<kFmt>(v.x, v.y, inv, max_fp8), q8x4<kFmt>(v.z, v.w, inv, max_fp8));
  }
  for (int64_t i = (nvec << 3) + threadIdx.x; i < n; i += kSmallThreads) {
    const float f = __half2float(x[i]);
    q[i] = static_cast<uint8_t>(q8x2<kFmt>(f, 0.0f, inv, max_fp8) & 0xFFu);
  }
}

// Register-resident variant for the smallest tensors (decoder-step activations,
// n <= 1024 threads x 10 x 8 elements): every thread issues all its 16-byte
// loads at once and keeps them in registers, so the tensor crosses memory once
// (one round trip of latency) instead of twice; same codes and scale.
constexpr int kRegVecs = 10;
constexpr int64_t kRegQuantMax = static_cast<int64_t>(kSmallThreads) * kRegVecs * 8;

template <int kFmt>
__global__ void __launch_bounds__(kSmallThreads, 1)
quantise_regs_kernel(const __half* __restrict__ x, int64_t n, float max_fp8, uint8_t* __restrict__ q,
                     float* __restrict__ scale_out, uint32_t* __restrict__ amax_out) {
  griddep_launch_dependents();  // a following GEMM may run its prologue meanwhile
  __shared__ uint32_t red[kSmallThreads / 32];
  __shared__ float sc[2];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nvec = static_cast<int>(n >> 3);
  const uint4* xv = reinterpret_cast<const uint4*>(x);
  uint4 v[kRegVecs];
#pragma unroll
  for (int k = 0; k < kRegVecs; ++k) {
    const int i = threadIdx.x + k * kSmallThreads;
    v[k] = i < nvec ? ld_stream16(xv + i) : make_uint4(0u, 0u, 0u, 0u);
  }
  uint32_t m = 0;
#pragma unroll
  for (int k = 0; k < kRegVecs; ++k)
    m = __vmaxu2(m, __vmaxu2(__vmaxu2(abs2_nonan(v[k].x), abs2_nonan(v[k].y)),
                             __vmaxu2(abs2_nonan(v[k].z), abs2_nonan(v[k].w))));
  uint32_t mm = warp_max_u32(max(m & 0xFFFFu, m >> 16));
  if (lane == 0) red[warp] = mm;
  __syncthreads();
  if (warp == 0) {
    mm = warp_max_u32(red[lane]);
    if (lane == 0) {
      float scale, inv;
      scale_from_amax(mm, max_fp8, scale, inv);
      sc[0] = scale;
      sc[1] = inv;
      if (scale_out != nullptr) *scale_out = scale;
      if (amax_out != nullptr) *amax_out = mm;
    }
  }
  __syncthreads();
  const float inv = sc[1];
  uint2* qv = reinterpret_cast<uint2*>(q);
#pragma unroll
  for (int k = 0; k < kRegVecs; ++k) {
    const int i = threadIdx.x + k * kSmallThreads;
    if (i < nvec) qv[i] = make_uint2(q8x4<kFmt>(v[k].x, v[k].y, inv, max_fp8), q8x4<kFmt>(v[k].z, v[k].w, inv, max_fp8));
  }
}

// -------------------------------------------------------------- dequantise

template <int kFmt>
__device__ __forceinline__ uint32_t dq8x2(uint32_t pair, float scale) {
  const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(pair & 0xFFFFu),
                                                    kFmt == WBK_FMT_E4M3 ? __NV_E4M3 : __NV_E5M2);
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hr));
  const __half2 o = __halves2half2(__float2half_rn(f.x * scale), __float2half_rn(f.y * scale));
  return *reinterpret_cast<const uint32_t*>(&o);
}

template <int kFmt, bool kVec>
__global__ void __launch_bounds__(kThreads)
dequantise_f16_kernel(const uint8_t* __restrict__ q, int64_t n, float scale, __half* __restrict__ out) {
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  int64_t done = 0;
  if (kVec) {
    const int64_t nvec = n >> 3;
    const uint2* qv = reinterpret_cast<const uint2*>(q);
    uint4* ov = reinterpret_cast<uint4*>(out);
    for (int64_t i = tid; i < nvec; i += stride) {
      const uint2 v = qv[i];
      ov[i] = make_uint4(dq8x2<kFmt>(v.x, scale), dq8x2<kFmt>(v.x >> 16, scale),
                         dq8x2<kFmt>(v.y, scale), dq8x2<kFmt>(v.y >> 16, scale));
    }
    done = nvec << 3;
  }
  for (int64_t i = done + tid; i < n; i += stride) {
    const uint32_t h = dq8x2<kFmt>(q[i], scale);
    reinterpret_cast<unsigned short*>(out)[i] = static_cast<unsigned short>(h & 0xFFFFu);
  }
}

int grid_for(int64_t work_items, int per_sm) {
  const int64_t want = (work_items + kThreads - 1) / kThreads;
  const int64_t cap = static_cast<int64_t>(sm_count() > 0 ? sm_count() : 148) * per_sm;
  const int64_t g = want < 1 ? 1 : (want < cap ? want : cap);
  return static_cast<int>(g);
}

int check_fmt(int fmt) {
  if (fmt != WBK_FMT_E4M3 && fmt != WBK_FMT_E5M2) return fail(WBK_ERR_INVALID_ARG, "unknown fp8 format %d", fmt);
  return WBK_OK;
}

// ------------------------------------------------- no-allocation quantise
//
// For callers that cannot allocate device memory themselves (code that runs
// where cudaMalloc is not allowed or not wanted, e.g. inside a host callback,
// a real-time audio thread with a no-allocation rule, or a plugin host that
// owns every device allocation), wbk_quantise_f16_noalloc keeps its scratch
// in this file-scope array instead of asking for an amax_ws buffer:
//   word 0           the tensor's amax (fp16 bits), written by the finalize kernel;
//   words 1..4095    one partial max per CTA of the amax pass, one CTA per
//                    kNoAllocElemsPerCta elements.
// Every GPU that loads libwbk holds these 16 KB until the process exits.
// Every word a call reads is written earlier in the same call, so nothing
// needs clearing; calls that overlap on the GPU (different streams at the
// same time) share the array and race.
constexpr int kNoAllocWords = 4096;
constexpr int kNoAllocMaxCtas = kNoAllocWords - 1;
constexpr int64_t kNoAllocElemsPerCta = 65536;  // 256 threads x 32 vectors of 8 halves
constexpr int64_t kNoAllocMaxElems = kNoAllocElemsPerCta * kNoAllocMaxCtas;
static __device__ __align__(256) uint32_t g_noalloc_scratch[kNoAllocWords];

// CTA b writes max|x| (fp16 bits, NaN ignored) over elements
// [b*kNoAllocElemsPerCta, (b+1)*kNoAllocElemsPerCta) to partials[b].
template <bool kVec>
__global__ void __launch_bounds__(kThreads)
amax_partials_kernel(const __half* __restrict__ x, int64_t n, uint32_t* __restrict__ partials) {
  const int64_t begin = static_cast<int64_t>(blockIdx.x) * kNoAllocElemsPerCta;
  const int64_t end = min(n, begin + kNoAllocElemsPerCta);
  uint32_t m = 0;
  int64_t done = begin;
  if (kVec) {
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    const int64_t vbegin = begin >> 3, vend = end >> 3;
    for (int64_t i = vbegin + threadIdx.x; i < vend; i += kThreads) {
      const uint4 v = ld_stream16(xv + i);
      m = __vmaxu2(m, __vmaxu2(__vmaxu2(abs2_nonan(v.x), abs2_nonan(v.y)),
                               __vmaxu2(abs2_nonan(v.z), abs2_nonan(v.w))));
    }
    done = vend << 3;
  }
  const unsigned short* xs = reinterpret_cast<const unsigned short*>(x);
  for (int64_t i = done + threadIdx.x; i < end; i += kThreads) m = __vmaxu2(m, abs2_nonan(xs[i]));
  uint32_t mm = warp_max_u32(max(m & 0xFFFFu, m >> 16));
  __shared__ uint32_t red[kThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = mm;
  __syncthreads();
  if (warp == 0) {
    mm = warp_max_u32(lane < kThreads / 32 ? red[lane] : 0u);
    if (lane == 0) partials[blockIdx.x] = mm;
  }
}

// One CTA: *amax_bits = max(partials[0..count)).
__global__ void __launch_bounds__(kThreads)
amax_finalize_kernel(const uint32_t* __restrict__ partials, int count, uint32_t* __restrict__ amax_bits) {
  uint32_t m = 0;
  for (int i = threadIdx.x; i < count; i += kThreads) m = max(m, partials[i]);
  m = warp_max_u32(m);
  __shared__ uint32_t red[kThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (warp == 0) {
    m = warp_max_u32(lane < kThreads / 32 ? red[lane] : 0u);
    if (lane == 0) *amax_bits = m;
  }
}

// The current CUDA context (driver cuCtxGetCurrent, fetched once through the
// runtime), or nullptr if none is current or the driver entry point is missing.
void* current_context() {
  using GetCtx = int (*)(void**);
  static std::once_flag once;
  static GetCtx fn = nullptr;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<GetCtx>(f);
  });
  void* ctx = nullptr;
  if (fn == nullptr || fn(&ctx) != 0) return nullptr;
  return ctx;
}

// Device address of g_noalloc_scratch for the current device. The host-side
// name is only a stand-in, so the address is looked up (with that device
// current) and cached per device together with the context it belongs to: a
// new context on the device (after cudaDeviceReset, the module is loaded
// again) makes the next call look the address up again.
int noalloc_scratch(uint32_t** out) {
  struct Entry {
    void* ctx = nullptr;
    uint32_t* ptr = nullptr;
  };
  static std::mutex mu;
  static std::vector<Entry> cache;
  const int dev = current_device();
  if (dev < 0) return fail(WBK_ERR_CUDA, "wbk_quantise_f16_noalloc: no current CUDA device");
  std::lock_guard<std::mutex> lock(mu);
  if (static_cast<int>(cache.size()) <= dev) cache.resize(dev + 1);
  Entry& e = cache[dev];
  void* ctx = current_context();
  if (e.ptr == nullptr || ctx == nullptr || ctx != e.ctx) {
    uint32_t* ptr = nullptr;
    // also makes the device's primary context current if nothing had yet
    if (int err = cuda_check(cudaGetSymbolAddress(reinterpret_cast<void**>(&ptr), g_noalloc_scratch),
                             "wbk_quantise_f16_noalloc: cudaGetSymbolAddress(scratch)"))
      return err;
    e.ptr = ptr;
    e.ctx = current_context();
  }
  *out = e.ptr;
  return WBK_OK;
}

}  // namespace
}  // namespace wbk

using namespace wbk;

extern "C" {

int wbk_amax_f16(const void* x, int64_t n, uint32_t* amax_bits, wbk_stream_t stream) {
  if (n < 0) return fail(WBK_ERR_INVALID_ARG, "wbk_amax_f16: n < 0");
  if (amax_bits == nullptr || (n > 0 && x == nullptr)) return fail(WBK_ERR_INVALID_ARG, "wbk_amax_f16: null pointer");
  if (n == 0) return WBK_OK;
  const bool vec = aligned(x, 16);
  const int grid = grid_for(vec ? (n + 7) / 8 / 4 : n, 8);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (vec) amax_f16_kernel<true><<<grid, kThreads, 0, s>>>(static_cast<const __half*>(x), n, amax_bits);
  else amax_f16_kernel<false><<<grid, kThreads, 0, s>>>(static_cast<const __half*>(x), n, amax_bits);
  return cuda_check(cudaGetLastError(), "wbk_amax_f16 launch");
}

int wbk_quantise_from_amax_f16(const void* x, int64_t n, int fmt, const uint32_t* amax_bits, void* q_out,
                               float* scale_out, wbk_stream_t stream) {
  if (int e = check_fmt(fmt)) return e;
  if (n < 0) return fail(WBK_ERR_INVALID_ARG, "wbk_quantise_from_amax_f16: n < 0");
  if (amax_bits == nullptr || (n > 0 && (x == nullptr || q_out == nullptr)))
    return fail(WBK_ERR_INVALID_ARG, "wbk_quantise_from_amax_f16: null pointer");
  const bool vec = aligned(x, 16) && aligned(q_out, 8);
  const int grid = grid_for(vec ? (n + 7) / 8 / 2 : n, 16);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const float mx = fmt_max(fmt);
  const __half* xh = static_cast<const __half*>(x);
  uint8_t* q = static_cast<uint8_t*>(q_out);
  if (fmt == WBK_FMT_E4M3) {
    if (vec) quantise_f16_kernel<WBK_FMT_E4M3, true><<<grid, kThreads, 0, s>>>(xh, n, amax_bits, mx, q, scale_out);
    else quantise_f16_kernel<WBK_FMT_E4M3, false><<<grid, kThreads, 0, s>>>(xh, n, amax_bits, mx, q, scale_out);
  } else {
    if (vec) quantise_f16_kernel<WBK_FMT_E5M2, true><<<grid, kThreads, 0, s>>>(xh, n, amax_bits, mx, q, scale_out);
    else quantise_f16_kernel<WBK_FMT_E5M2, false><<<grid, kThreads, 0, s>>>(xh, n, amax_bits, mx, q, scale_out);
  }
  return cuda_check(cudaGetLastError(), "wbk_quantise_from_amax_f16 launch");
}

int wbk_quantise_f16(const void* x, int64_t n, int fmt, void* q_out, float* scale_out, uint32_t* amax_ws,
                     wbk_stream_t stream) {
  if (int e = check_fmt(fmt)) return e;
  if (amax_ws == nullptr) return fail(WBK_ERR_INVALID_ARG, "wbk_quantise_f16: amax_ws is null");
  if (n < 0) return fail(WBK_ERR_INVALID_ARG, "wbk_quantise_f16: n < 0");
  if (n > 0 && (x == nullptr || q_out == nullptr)) return fail(WBK_ERR_INVALID_ARG, "wbk_quantise_f16: null pointer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (n <= kSmallQuantMax) {  // one launch; *amax_ws receives the amax as in the general path
    const bool vec = aligned(x, 16) && aligned(q_out, 8);
    const __half* xh = static_cast<const __half*>(x);
    uint8_t* q = static_cast<uint8_t*>(q_out);
    const float mx = fmt_max(fmt);
    if (vec && n % 8 == 0 && n <= kRegQuantMax) {
      if (fmt == WBK_FMT_E4M3) quantise_regs_kernel<WBK_FMT_E4M3><<<1, kSmallThreads, 0, s>>>(xh, n, mx, q, scale_out, amax_ws);
      else quantise_regs_kernel<WBK_FMT_E5M2><<<1, kSmallThreads, 0, s>>>(xh, n, mx, q, scale_out, amax_ws);
      return cuda_check(cudaGetLastError(), "wbk_quantise_f16 (small, registers) launch");
    }
    if (fmt == WBK_FMT_E4M3) {
      if (vec) quantise_small_kernel<WBK_FMT_E4M3, true><<<1, kSmallThreads, 0, s>>>(xh, n, mx, q, scale_out, amax_ws);
      else quantise_small_kernel<WBK_FMT_E4M3, false><<<1, kSmallThreads, 0, s>>>(xh, n, mx, q, scale_out, amax_ws);
    } else {
      if (vec) quantise_small_kernel<WBK_FMT_E5M2, true><<<1, kSmallThreads, 0, s>>>(xh, n, mx, q, scale_out, amax_ws);
      else quantise_small_kernel<WBK_FMT_E5M2, false><<<1, kSmallThreads, 0, s>>>(xh, n, mx, q, scale_out, amax_ws);
    }
    return cuda_check(cudaGetLastError(), "wbk_quantise_f16 (small) launch");
  }
  if (int e = cuda_check(cudaMemsetAsync(amax_ws, 0, sizeof(uint32_t), s), "wbk_quantise_f16 memset")) return e;
  if (int e = wbk_amax_f16(x, n, amax_ws, stream)) return e;
  return wbk_quantise_from_amax_f16(x, n, fmt, amax_ws, q_out, scale_out, stream);
}

int wbk_scale_from_amax(const uint32_t* amax_bits, int fmt, float* scale_inv, wbk_stream_t stream) {
  if (int e = check_fmt(fmt)) return e;
  if (amax_bits == nullptr || scale_inv == nullptr) return fail(WBK_ERR_INVALID_ARG, "wbk_scale_from_amax: null pointer");
  scale_from_amax_kernel<<<1, 1, 0, reinterpret_cast<cudaStream_t>(stream)>>>(amax_bits, fmt_max(fmt), scale_inv);
  return cuda_check(cudaGetLastError(), "wbk_scale_from_amax launch");
}

int wbk_quantise_gelu_f16(const void* y, int64_t n, int fmt, const uint32_t* ymax_key, void* q_out,
                          float* scale_out, uint32_t* amax_ws, wbk_stream_t stream) {
  if (int e = check_fmt(fmt)) return e;
  if (amax_ws == nullptr) return fail(WBK_ERR_INVALID_ARG, "wbk_quantise_gelu_f16: amax_ws is null");
  if (n < 0) return fail(WBK_ERR_INVALID_ARG, "wbk_quantise_gelu_f16: n < 0");
  if (n > 0 && (y == nullptr || q_out == nullptr)) return fail(WBK_ERR_INVALID_ARG, "wbk_quantise_gelu_f16: null pointer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const __half* yh = static_cast<const __half*>(y);
  if (int e = cuda_check(cudaMemsetAsync(amax_ws, 0, sizeof(uint32_t), s), "wbk_quantise_gelu_f16 memset")) return e;
  const bool vec = aligned(y, 16) && aligned(q_out, 8);
  const int agrid = grid_for(vec ? (n + 7) / 8 : n, 8);
  if (vec) gelu_amax_kernel<true><<<agrid, kThreads, 0, s>>>(yh, n, ymax_key, amax_ws);
  else gelu_amax_kernel<false><<<agrid, kThreads, 0, s>>>(yh, n, ymax_key, amax_ws);
  if (int e = cuda_check(cudaGetLastError(), "wbk_quantise_gelu_f16 amax launch")) return e;
  const float mx = fmt_max(fmt);
  uint8_t* q = static_cast<uint8_t*>(q_out);
  if (fmt == WBK_FMT_E4M3)
    return vec ? launch_quantise_gelu<WBK_FMT_E4M3, true>(yh, n, amax_ws, mx, q, scale_out, s)
               : launch_quantise_gelu<WBK_FMT_E4M3, false>(yh, n, amax_ws, mx, q, scale_out, s);
  return vec ? launch_quantise_gelu<WBK_FMT_E5M2, true>(yh, n, amax_ws, mx, q, scale_out, s)
             : launch_quantise_gelu<WBK_FMT_E5M2, false>(yh, n, amax_ws, mx, q, scale_out, s);
}

int wbk_dequantise_f16(const void* q, int64_t n, int fmt, float scale, void* out, wbk_stream_t stream) {
  if (int e = check_fmt(fmt)) return e;
  if (n < 0) return fail(WBK_ERR_INVALID_ARG, "wbk_dequantise_f16: n < 0");
  if (n == 0) return WBK_OK;
  if (q == nullptr || out == nullptr) return fail(WBK_ERR_INVALID_ARG, "wbk_dequantise_f16: null pointer");
  const bool vec = aligned(q, 8) && aligned(out, 16);
  const int grid = grid_for(vec ? (n + 7) / 8 : n, 16);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const uint8_t* qq = static_cast<const uint8_t*>(q);
  __half* o = static_cast<__half*>(out);
  if (fmt == WBK_FMT_E4M3) {
    if (vec) dequantise_f16_kernel<WBK_FMT_E4M3, true><<<grid, kThreads, 0, s>>>(qq, n, scale, o);
    else dequantise_f16_kernel<WBK_FMT_E4M3, false><<<grid, kThreads, 0, s>>>(qq, n, scale, o);
  } else {
    if (vec) dequantise_f16_kernel<WBK_FMT_E5M2, true><<<grid, kThreads, 0, s>>>(qq, n, scale, o);
    else dequantise_f16_kernel<WBK_FMT_E5M2, false><<<grid, kThreads, 0, s>>>(qq, n, scale, o);
  }
  return cuda_check(cudaGetLastError(), "wbk_dequantise_f16 launch");
}

int wbk_quantise_f16_noalloc(const void* x, int64_t n, int fmt, void* q_out, float* scale_out,
                             wbk_stream_t stream) {
  if (int e = check_fmt(fmt)) return e;
  if (n < 0) return fail(WBK_ERR_INVALID_ARG, "wbk_quantise_f16_noalloc: n < 0");
  if (n > kNoAllocMaxElems)
    return fail(WBK_ERR_UNSUPPORTED,
                "wbk_quantise_f16_noalloc: n = %lld elements exceeds the limit of %lld set by its static scratch "
                "(%d words); use wbk_quantise_f16 with a caller-provided amax_ws for larger tensors",
                (long long)n, (long long)kNoAllocMaxElems, kNoAllocWords);
  if (n > 0 && (x == nullptr || q_out == nullptr))
    return fail(WBK_ERR_INVALID_ARG, "wbk_quantise_f16_noalloc: null pointer");
  uint32_t* scratch = nullptr;
  if (int e = noalloc_scratch(&scratch)) return e;
  uint32_t* amax_word = scratch;
  uint32_t* partials = scratch + 1;
  const int ctas = static_cast<int>(n == 0 ? 1 : (n + kNoAllocElemsPerCta - 1) / kNoAllocElemsPerCta);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const __half* xh = static_cast<const __half*>(x);
  if (aligned(x, 16)) amax_partials_kernel<true><<<ctas, kThreads, 0, s>>>(xh, n, partials);
  else amax_partials_kernel<false><<<ctas, kThreads, 0, s>>>(xh, n, partials);
  if (int e = cuda_check(cudaGetLastError(), "wbk_quantise_f16_noalloc amax launch")) return e;
  amax_finalize_kernel<<<1, kThreads, 0, s>>>(partials, ctas, amax_word);
  if (int e = cuda_check(cudaGetLastError(), "wbk_quantise_f16_noalloc finalize launch")) return e;
  return wbk_quantise_from_amax_f16(x, n, fmt, amax_word, q_out, scale_out, stream);
}

}  // extern "C"
