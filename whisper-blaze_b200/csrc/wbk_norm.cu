// Fused residual-add + LayerNorm / RMSNorm for B200.
//
// Semantics follow the reference's layernorm_fused_kernel and
// rmsnorm_fused_kernel (csrc/kernels/layernorm_fused.cu:50-184, :191-258):
// s = float(x) (+ float(residual)); mean and variance in fp32 (two passes over
// the row, the second over (s - mean)); out = fp16((s - mean) * rsqrt(var + eps)
// * gamma + beta); the optional sum output is fp16(s).
//
// Design: one warp per row with the whole row held in registers (D <= 4096),
// so x and residual are read from HBM exactly once — the reference reads them
// three times, one CTA per row. Rows are strided over a persistent grid so the
// optional output-amax (for a following FP8 quantise without another pass)
// costs one atomic per CTA. Rows with D > 4096 use a CTA-per-row kernel that
// re-reads the row (served from L2).
#include "wbk_common.cuh"
#include "wbk_fp8_quant.cuh"

namespace wbk {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

__device__ __forceinline__ void unpack8(const uint4& v, float* f) {
  const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 t = __half22float2(h[j]);
    f[2 * j] = t.x;
    f[2 * j + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float* f) {
  uint4 r;
  uint32_t* w = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __half2 h = __halves2half2(__float2half_rn(f[2 * j]), __float2half_rn(f[2 * j + 1]));
    w[j] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return r;
}

__device__ __forceinline__ uint32_t amax8(const uint4& v) {
  const uint32_t m = __vmaxu2(__vmaxu2(abs2_nonan(v.x), abs2_nonan(v.y)), __vmaxu2(abs2_nonan(v.z), abs2_nonan(v.w)));
  return max(m & 0xFFFFu, m >> 16);
}

__device__ __forceinline__ void block_amax_commit(uint32_t m, uint32_t* out_amax) {
  __shared__ uint32_t red[kWarps];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  m = warp_max_u32(m);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (warp == 0) {
    m = lane < kWarps ? red[lane] : 0u;
    m = warp_max_u32(m);
    if (lane == 0 && m != 0u) atomicMax(out_amax, m);
  }
}

// Per-row pieces shared by every mode of norm_warp_kernel, so the stats-only
// pass and the quantise pass of the fused LayerNorm->FP8 path compute exactly
// the same fp16 outputs as the plain LayerNorm.
// kRes = false: the residual operand is known to be absent at compile time and
// its registers are not allocated.
template <int kVpl, bool kRes>
__device__ __forceinline__ void load_row_raw(const uint4* xr, const uint4* rr, int lane, int nvec, uint4 (&xv)[kVpl],
                                             uint4 (&rv)[kVpl]) {
#pragma unroll
  for (int i = 0; i < kVpl; ++i) {
    const int idx = lane + 32 * i;
    xv[i] = idx < nvec ? ld_stream16(xr + idx) : make_uint4(0, 0, 0, 0);
    if (kRes && rr) rv[i] = idx < nvec ? ld_stream16(rr + idx) : make_uint4(0, 0, 0, 0);
  }
}

template <int kVpl, bool kRes>
__device__ __forceinline__ void unpack_row(const uint4 (&xv)[kVpl], const uint4 (&rv)[kVpl], bool has_res,
                                           float (&v)[kVpl][8]) {
#pragma unroll
  for (int i = 0; i < kVpl; ++i) {
    unpack8(xv[i], v[i]);
    if (kRes && has_res) {
      float r8[8];
      unpack8(rv[i], r8);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] += r8[j];
    }
  }
}

// Row statistics. LayerNorm leaves v[i][j] - mean in v (the same fp32 value
// the normalisation subtracts), so normalise8 takes centred values.
template <int kVpl, bool kRms>
__device__ __forceinline__ void row_stats(float (&v)[kVpl][8], int lane, int nvec, float fD, float eps, float& mean,
                                          float& inv) {
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < kVpl; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) s += kRms ? v[i][j] * v[i][j] : v[i][j];
  s = warp_sum(s);
  if (kRms) {
    mean = 0.0f;
    inv = rsqrtf(s / fD + eps);
    return;
  }
  mean = s / fD;
  float var = 0.0f;
  const float2 neg_mean = make_float2(-mean, -mean);
#pragma unroll
  for (int i = 0; i < kVpl; ++i) {
#pragma unroll
    for (int j = 0; j < 8; j += 2) {  // v - mean, two lanes per instruction
      const float2 d = f2_add(make_float2(v[i][j], v[i][j + 1]), neg_mean);
      v[i][j] = d.x;
      v[i][j + 1] = d.y;
    }
    if (lane + 32 * i < nvec) {
#pragma unroll
      for (int j = 0; j < 8; ++j) var += v[i][j] * v[i][j];
    }
  }
  var = warp_sum(var);
  inv = rsqrtf(var / fD + eps);
}

// fp32 outputs before the fp16 rounding: LayerNorm fma(d * inv, gamma, beta)
// with d = s - mean, RMSNorm (s * inv) * gamma.
template <bool kRms>
__device__ __forceinline__ void normalise8(const float* d8, int idx, const __half* __restrict__ gamma,
                                           const __half* __restrict__ beta, float inv, float* o) {
  float g[8];
  unpack8(__ldg(reinterpret_cast<const uint4*>(gamma) + idx), g);
  if (kRms) {
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = (d8[j] * inv) * g[j];
  } else {
    float b[8];
    unpack8(__ldg(reinterpret_cast<const uint4*>(beta) + idx), b);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = fmaf(d8[j] * inv, g[j], b[j]);
  }
}

// max |o| over 8 fp32 outputs; NaN is skipped (fmaxf), as abs2_nonan skips it
// in the fp16 amax. Rounding to fp16 is monotone and symmetric, so
// fp16(max|o|) equals the max of |fp16(o)|: the amax of the stored outputs.
__device__ __forceinline__ float absmax8(const float* o, float m) {
#pragma unroll
  for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(o[j]));
  return m;
}

enum NormMode { kModeNormal = 0, kModeStats = 1, kModeQuant = 2 };

// kVpl = 16-byte vectors (8 halves) per lane; the row has D/8 vectors.
//   kModeNormal: out (+ sum_out, + out_amax) as wbk_layernorm_f16 / wbk_rmsnorm_f16;
//   kModeStats:  stats[row] = (mean, rstd) and out_amax of the fp16 outputs, nothing else stored;
//   kModeQuant:  fp8 codes of the fp16 outputs, from stats[] and the scale of the statistics pass's
//                amax (*out_amax), which CTA 0 also stores to scale_inv = (scale, 1/scale) and scale_out.
// Rows up to 1536 wide (kVpl <= 6) run two CTAs per SM; without a residual
// operand they are also software-pipelined (two rows in flight per warp).
template <int kVpl, bool kRms, int kMode, int kFmt>
__global__ void __launch_bounds__(kThreads, kVpl <= 6 ? 2 : 1)
norm_warp_kernel(const __half* __restrict__ x, const __half* __restrict__ res, const __half* __restrict__ gamma,
                 const __half* __restrict__ beta, __half* __restrict__ out, __half* __restrict__ sum_out,
                 int64_t rows, int D, float eps, uint32_t* __restrict__ out_amax, float2* __restrict__ stats,
                 float* __restrict__ scale_inv, uint8_t* __restrict__ q_out, float* __restrict__ scale_out) {
  griddep_launch_dependents();  // a following GEMM may run its prologue meanwhile
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nvec = D >> 3;
  const float fD = static_cast<float>(D);
  // The fused LayerNorm->FP8 passes are issue-bound; gamma and beta are the same for
  // every row, so they are converted to fp32 once per CTA into shared memory instead
  // of being reloaded and unpacked for each row (the same fp32 values, so the outputs
  // do not change). Layout [gamma lo, gamma hi, beta lo, beta hi][vector]: a warp's
  // 16-byte reads of consecutive vectors are conflict-free.
  constexpr bool kGbShared = kMode != kModeNormal;
  __shared__ float4 s_gb[kGbShared ? 4 : 1][kGbShared ? kVpl * 32 : 1];
  if constexpr (kGbShared) {
    for (int idx = threadIdx.x; idx < nvec; idx += kThreads) {
      float g[8], b[8];
      unpack8(__ldg(reinterpret_cast<const uint4*>(gamma) + idx), g);
      unpack8(__ldg(reinterpret_cast<const uint4*>(beta) + idx), b);
      s_gb[0][idx] = make_float4(g[0], g[1], g[2], g[3]);
      s_gb[1][idx] = make_float4(g[4], g[5], g[6], g[7]);
      s_gb[2][idx] = make_float4(b[0], b[1], b[2], b[3]);
      s_gb[3][idx] = make_float4(b[4], b[5], b[6], b[7]);
    }
    __syncthreads();
  }
  float amax_f = 0.0f;
  float qinv = 0.0f;
  constexpr float kMx = kFmt == WBK_FMT_E4M3 ? 448.0f : 57344.0f;
  if (kMode == kModeQuant) {
    // The quantiser's scale rule on the amax (the same device function as the scale kernels), so no
    // separate launch computes it between the two passes.
    float sc;
    scale_from_amax(*out_amax, kMx, sc, qinv);
    if (blockIdx.x == 0 && threadIdx.x == 0) {
      if (scale_out != nullptr) *scale_out = sc;
      scale_inv[0] = sc;
      scale_inv[1] = qinv;
    }
  }
  // Rows are software-pipelined: the loads of this warp's next row are issued
  // before the current row's reductions, so each warp keeps a row in flight.
  constexpr bool kRes = kMode == kModeNormal;  // the fused LayerNorm->FP8 passes take no residual
  auto process_row = [&](int64_t row, const uint4 (&xv)[kVpl], const uint4 (&rv)[kVpl]) {
    float v[kVpl][8];
    unpack_row<kVpl, kRes>(xv, rv, res != nullptr, v);
    if (kMode == kModeNormal && sum_out) {  // fp16(s), before LayerNorm centres v
#pragma unroll
      for (int i = 0; i < kVpl; ++i)
        if (lane + 32 * i < nvec) reinterpret_cast<uint4*>(sum_out + row * D)[lane + 32 * i] = pack8(v[i]);
    }
    float mean, inv;
    if (kMode == kModeQuant) {
      const float2 st = stats[row];
      mean = st.x;
      inv = st.y;
      const float2 neg_mean = make_float2(-mean, -mean);
#pragma unroll
      for (int i = 0; i < kVpl; ++i)
#pragma unroll
        for (int j = 0; j < 8; j += 2) {  // v - mean, two lanes per instruction
          const float2 d = f2_add(make_float2(v[i][j], v[i][j + 1]), neg_mean);
          v[i][j] = d.x;
          v[i][j + 1] = d.y;
        }
    } else {
      row_stats<kVpl, kRms>(v, lane, nvec, fD, eps, mean, inv);
      if (kMode == kModeStats && lane == 0) stats[row] = make_float2(mean, inv);
    }
#pragma unroll
    for (int i = 0; i < kVpl; ++i) {
      const int idx = lane + 32 * i;
      if (idx < nvec) {
        float o[8];
        if constexpr (kGbShared) {
          // fma(d * inv, gamma, beta): the expression normalise8 evaluates, on the staged
          // values, two lanes per instruction (each lane rounded as the scalar form)
          const float4 g0 = s_gb[0][idx], g1 = s_gb[1][idx], b0 = s_gb[2][idx], b1 = s_gb[3][idx];
          const float2 g[4] = {make_float2(g0.x, g0.y), make_float2(g0.z, g0.w), make_float2(g1.x, g1.y),
                               make_float2(g1.z, g1.w)};
          const float2 bb[4] = {make_float2(b0.x, b0.y), make_float2(b0.z, b0.w), make_float2(b1.x, b1.y),
                                make_float2(b1.z, b1.w)};
          const float2 inv2 = make_float2(inv, inv);
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const float2 r = f2_fma(f2_mul(make_float2(v[i][2 * t], v[i][2 * t + 1]), inv2), g[t], bb[t]);
            o[2 * t] = r.x;
            o[2 * t + 1] = r.y;
          }
        } else {
          normalise8<kRms>(v[i], idx, gamma, beta, inv, o);
        }
        if (kMode != kModeQuant && out_amax) amax_f = absmax8(o, amax_f);
        if (kMode == kModeNormal) reinterpret_cast<uint4*>(out + row * D)[idx] = pack8(o);
        if (kMode == kModeQuant && qinv != 0.0f) {
          // fp8(fp16(o) * (1/scale)) by q8x4_fin (qinv is finite and > 0 here), the
          // quantiser's element rule on the fp16 outputs.
          uint32_t h[4];
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const __half2 hh = __floats2half2_rn(o[2 * t], o[2 * t + 1]);
            h[t] = *reinterpret_cast<const uint32_t*>(&hh);
          }
          reinterpret_cast<uint2*>(q_out + row * D)[idx] =
              make_uint2(q8x4_fin<kFmt>(h[0], h[1], qinv), q8x4_fin<kFmt>(h[2], h[3], qinv));
        } else if (kMode == kModeQuant) {
          // An infinite amax (qinv = 0): fp8(fp16(o) * (1/scale)) where fmaxf maps NaN
          // to -max as the quantiser's clamp does; satfinite clamps everything else to +-max.
          uint32_t q[2];
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const float2 f0 = __half22float2(__floats2half2_rn(o[4 * t], o[4 * t + 1]));
            const float2 f1 = __half22float2(__floats2half2_rn(o[4 * t + 2], o[4 * t + 3]));
            float2 c0, c1;
            c0.x = fmaxf(f0.x * qinv, -kMx);
            c0.y = fmaxf(f0.y * qinv, -kMx);
            c1.x = fmaxf(f1.x * qinv, -kMx);
            c1.y = fmaxf(f1.y * qinv, -kMx);
            const __nv_fp8_interpretation_t it = kFmt == WBK_FMT_E4M3 ? __NV_E4M3 : __NV_E5M2;
            q[t] = static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(c0, __NV_SATFINITE, it)) |
                   (static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(c1, __NV_SATFINITE, it)) << 16);
          }
          reinterpret_cast<uint2*>(q_out + row * D)[idx] = make_uint2(q[0], q[1]);
        }
      }
    }
  };
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kWarps;
  int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + warp;
  // The quantise pass visits rows last to first: the statistics pass that ran
  // just before read them first to last, so the rows still in L2 come first.
  auto phys = [&](int64_t r) { return kMode == kModeQuant ? rows - 1 - r : r; };
  auto row_ptrs = [&](int64_t r, const uint4*& xr, const uint4*& rr) {
    const int64_t pr = phys(r);
    xr = reinterpret_cast<const uint4*>(x + pr * D);
    rr = res ? reinterpret_cast<const uint4*>(res + pr * D) : nullptr;
  };
  uint4 xa[kVpl], ra[kVpl], xb[kVpl], rb[kVpl];
  const uint4 *xr, *rr;
  if (kVpl > 6 || (kRes && res != nullptr)) {  // one row in flight per warp
    for (; row < rows; row += stride) {
      row_ptrs(row, xr, rr);
      load_row_raw<kVpl, kRes>(xr, rr, lane, nvec, xa, ra);
      process_row(phys(row), xa, ra);
    }
  } else {
    if (row < rows) {
      row_ptrs(row, xr, rr);
      load_row_raw<kVpl, kRes>(xr, rr, lane, nvec, xa, ra);
    }
    while (row < rows) {
      int64_t next = row + stride;
      if (next < rows) {
        row_ptrs(next, xr, rr);
        load_row_raw<kVpl, kRes>(xr, rr, lane, nvec, xb, rb);
      }
      process_row(phys(row), xa, ra);
      row = next;
      if (row >= rows) break;
      next = row + stride;
      if (next < rows) {
        row_ptrs(next, xr, rr);
        load_row_raw<kVpl, kRes>(xr, rr, lane, nvec, xa, ra);
      }
      process_row(phys(row), xb, rb);
      row = next;
    }
  }
  if (kMode != kModeQuant && out_amax)
    block_amax_commit(static_cast<uint32_t>(__half_as_ushort(__float2half_rn(amax_f))), out_amax);
}

// One wave of norm_warp_kernel: resident CTAs per SM (from the occupancy
// calculator, once per instantiation) x SMs, fewer when there are fewer rows.
template <int kVpl, bool kRms, int kMode, int kFmt>
int norm_warp_grid(int64_t rows) {
  static const int per_sm = [] {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, norm_warp_kernel<kVpl, kRms, kMode, kFmt>, kThreads, 0) !=
            cudaSuccess || n < 1) {
      (void)cudaGetLastError();
      n = 1;
    }
    return n;
  }();
  const int sms = sm_count() > 0 ? sm_count() : 148;
  const int64_t want = (rows + kWarps - 1) / kWarps;
  const int64_t cap = static_cast<int64_t>(sms) * per_sm;
  return static_cast<int>(want < cap ? want : cap);
}

// CTA per row, for D > 32*8*16. Three reads of the row (L2-resident).
template <bool kRms>
__global__ void __launch_bounds__(kThreads)
norm_block_kernel(const __half* __restrict__ x, const __half* __restrict__ res, const __half* __restrict__ gamma,
                  const __half* __restrict__ beta, __half* __restrict__ out, __half* __restrict__ sum_out,
                  int64_t rows, int D, float eps, uint32_t* __restrict__ out_amax) {
  __shared__ float red[kWarps];
  __shared__ float bcast;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nvec = D >> 3;
  const float fD = static_cast<float>(D);
  uint32_t amax = 0;
  auto block_sum = [&](float v) -> float {
    v = warp_sum(v);
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
      v = lane < kWarps ? red[lane] : 0.0f;
      v = warp_sum(v);
      if (lane == 0) bcast = v;
    }
    __syncthreads();
    const float r = bcast;
    __syncthreads();  // red/bcast are reused by the next reduction
    return r;
  };
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + row * D);
    const uint4* rr = res ? reinterpret_cast<const uint4*>(res + row * D) : nullptr;
    auto load = [&](int idx, float* f) {
      unpack8(xr[idx], f);
      if (rr) {
        float r8[8];
        unpack8(rr[idx], r8);
#pragma unroll
        for (int j = 0; j < 8; ++j) f[j] += r8[j];
      }
    };
    float s = 0.0f;
    for (int idx = threadIdx.x; idx < nvec; idx += kThreads) {
      float f[8];
      load(idx, f);
#pragma unroll
      for (int j = 0; j < 8; ++j) s += kRms ? f[j] * f[j] : f[j];
    }
    s = block_sum(s);
    float mean = 0.0f, inv;
    if (kRms) {
      inv = rsqrtf(s / fD + eps);
    } else {
      mean = s / fD;
      float var = 0.0f;
      for (int idx = threadIdx.x; idx < nvec; idx += kThreads) {
        float f[8];
        load(idx, f);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float d = f[j] - mean;
          var += d * d;
        }
      }
      var = block_sum(var);
      inv = rsqrtf(var / fD + eps);
    }
    for (int idx = threadIdx.x; idx < nvec; idx += kThreads) {
      float f[8], g[8], o[8];
      load(idx, f);
      unpack8(reinterpret_cast<const uint4*>(gamma)[idx], g);
      if (kRms) {
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = (f[j] * inv) * g[j];
      } else {
        float b[8];
        unpack8(reinterpret_cast<const uint4*>(beta)[idx], b);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = ((f[j] - mean) * inv) * g[j] + b[j];
      }
      const uint4 ov = pack8(o);
      reinterpret_cast<uint4*>(out + row * D)[idx] = ov;
      if (out_amax) amax = max(amax, amax8(ov));
      if (sum_out) reinterpret_cast<uint4*>(sum_out + row * D)[idx] = pack8(f);
    }
  }
  if (out_amax) block_amax_commit(amax, out_amax);
}

template <bool kRms>
int launch_norm(const void* x, const void* res, const void* gamma, const void* beta, void* out, void* sum_out,
                int64_t rows, int64_t D, float eps, uint32_t* out_amax, cudaStream_t s) {
  const __half* xh = static_cast<const __half*>(x);
  const __half* rh = static_cast<const __half*>(res);
  const __half* gh = static_cast<const __half*>(gamma);
  const __half* bh = static_cast<const __half*>(beta);
  __half* oh = static_cast<__half*>(out);
  __half* sh = static_cast<__half*>(sum_out);
  const int d = static_cast<int>(D);
  const int nvec = d / 8;
  const int sms = sm_count() > 0 ? sm_count() : 148;
#define WBK_NORM_CASE(V)                                                                       \
  if (nvec <= 32 * (V)) {                                                                      \
    const int grid = norm_warp_grid<V, kRms, kModeNormal, 0>(rows);                            \
    norm_warp_kernel<V, kRms, kModeNormal, 0><<<grid, kThreads, 0, s>>>(xh, rh, gh, bh, oh, sh, rows, d, eps,  \
                                                                      out_amax, nullptr, nullptr, nullptr, nullptr); \
    return cuda_check(cudaGetLastError(), "norm kernel launch");                               \
  }
  WBK_NORM_CASE(1)
  WBK_NORM_CASE(2)
  WBK_NORM_CASE(3)
  WBK_NORM_CASE(4)
  WBK_NORM_CASE(5)
  WBK_NORM_CASE(6)
  WBK_NORM_CASE(8)
  WBK_NORM_CASE(12)
  WBK_NORM_CASE(16)
#undef WBK_NORM_CASE
  const int bgrid = static_cast<int>(rows < sms * 8 ? rows : sms * 8);
  norm_block_kernel<kRms><<<bgrid, kThreads, 0, s>>>(xh, rh, gh, bh, oh, sh, rows, d, eps, out_amax);
  return cuda_check(cudaGetLastError(), "norm kernel launch");
}

// Fused LayerNorm -> FP8 quantise, D <= 32*8*16 (warp-per-row kernel only, so
// the stats pass and the quantise pass run the same per-row arithmetic).
template <int kMode, int kFmt>
int launch_ln_mode(const __half* x, const __half* gamma, const __half* beta, int64_t rows, int D, float eps,
                   uint32_t* amax, float2* stats, float* scale_inv, uint8_t* q, float* scale_out, cudaStream_t s) {
  const int nvec = D / 8;
#define WBK_LNQ_CASE(V)                                                                                  \
  if (nvec <= 32 * (V)) {                                                                                \
    const int grid = norm_warp_grid<V, false, kMode, kFmt>(rows);                                       \
    norm_warp_kernel<V, false, kMode, kFmt><<<grid, kThreads, 0, s>>>(x, nullptr, gamma, beta, nullptr, \
                                                                      nullptr, rows, D, eps, amax,       \
                                                                      stats, scale_inv, q, scale_out);   \
    return cuda_check(cudaGetLastError(), "layernorm-quantise launch");                                 \
  }
  WBK_LNQ_CASE(1)
  WBK_LNQ_CASE(2)
  WBK_LNQ_CASE(3)
  WBK_LNQ_CASE(4)
  WBK_LNQ_CASE(5)
  WBK_LNQ_CASE(6)
  WBK_LNQ_CASE(8)
  WBK_LNQ_CASE(12)
  WBK_LNQ_CASE(16)
#undef WBK_LNQ_CASE
  return fail(WBK_ERR_UNSUPPORTED, "wbk_layernorm_quantise_f16: D=%d exceeds 4096", D);
}

int check_norm_args(const char* who, const void* x, const void* res, const void* gamma, const void* beta, const void* out,
                    const void* sum_out, int64_t rows, int64_t D, bool need_beta) {
  if (rows < 0 || D <= 0) return fail(WBK_ERR_INVALID_ARG, "%s: rows=%lld D=%lld", who, (long long)rows, (long long)D);
  if (D % 8 != 0) return fail(WBK_ERR_UNSUPPORTED, "%s: last dimension %lld is not a multiple of 8", who, (long long)D);
  if (D > (int64_t(1) << 30)) return fail(WBK_ERR_UNSUPPORTED, "%s: last dimension too large", who);
  if (x == nullptr || gamma == nullptr || out == nullptr || (need_beta && beta == nullptr))
    return fail(WBK_ERR_INVALID_ARG, "%s: null pointer", who);
  const void* ptrs[6] = {x, res, gamma, beta, out, sum_out};
  for (const void* p : ptrs)
    if (p != nullptr && !aligned(p, 16)) return fail(WBK_ERR_UNSUPPORTED, "%s: pointer %p is not 16-byte aligned", who, p);
  return WBK_OK;
}

}  // namespace
}  // namespace wbk

using namespace wbk;

extern "C" {

int wbk_layernorm_f16(const void* x, const void* residual, const void* gamma, const void* beta, void* out,
                      void* sum_out, int64_t rows, int64_t D, float eps, uint32_t* out_amax_bits,
                      wbk_stream_t stream) {
  if (int e = check_norm_args("wbk_layernorm_f16", x, residual, gamma, beta, out, sum_out, rows, D, true)) return e;
  if (rows == 0) return WBK_OK;
  return launch_norm<false>(x, residual, gamma, beta, out, sum_out, rows, D, eps, out_amax_bits,
                            reinterpret_cast<cudaStream_t>(stream));
}

int wbk_rmsnorm_f16(const void* x, const void* residual, const void* gamma, void* out, int64_t rows, int64_t D,
                    float eps, wbk_stream_t stream) {
  if (residual == nullptr) return fail(WBK_ERR_INVALID_ARG, "wbk_rmsnorm_f16: residual is required");
  if (int e = check_norm_args("wbk_rmsnorm_f16", x, residual, gamma, nullptr, out, nullptr, rows, D, false)) return e;
  if (rows == 0) return WBK_OK;
  return launch_norm<true>(x, residual, gamma, nullptr, out, nullptr, rows, D, eps, nullptr,
                           reinterpret_cast<cudaStream_t>(stream));
}

int64_t wbk_layernorm_quantise_ws_bytes(int64_t rows) {
  return (rows > 0 ? rows : 0) * static_cast<int64_t>(sizeof(float2)) + 16;
}

int wbk_layernorm_quantise_f16(const void* x, const void* gamma, const void* beta, int64_t rows, int64_t D, float eps,
                               int fmt, void* q_out, float* scale_out, void* ws, uint32_t* amax_ws,
                               wbk_stream_t stream) {
  if (fmt != WBK_FMT_E4M3 && fmt != WBK_FMT_E5M2)
    return fail(WBK_ERR_INVALID_ARG, "wbk_layernorm_quantise_f16: unknown fp8 format %d", fmt);
  if (int e = check_norm_args("wbk_layernorm_quantise_f16", x, nullptr, gamma, beta, q_out, nullptr, rows, D, true))
    return e;
  if (D > 4096) return fail(WBK_ERR_UNSUPPORTED, "wbk_layernorm_quantise_f16: D=%lld exceeds 4096", (long long)D);
  if (ws == nullptr || amax_ws == nullptr) return fail(WBK_ERR_INVALID_ARG, "wbk_layernorm_quantise_f16: null workspace");
  if (!aligned(ws, 16)) return fail(WBK_ERR_INVALID_ARG, "wbk_layernorm_quantise_f16: ws must be 16-byte aligned");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  float2* stats = static_cast<float2*>(ws);
  float* scale_inv = reinterpret_cast<float*>(static_cast<char*>(ws) + rows * sizeof(float2));
  if (int e = cuda_check(cudaMemsetAsync(amax_ws, 0, sizeof(uint32_t), s), "wbk_layernorm_quantise_f16 memset"))
    return e;
  const __half* xh = static_cast<const __half*>(x);
  const __half* gh = static_cast<const __half*>(gamma);
  const __half* bh = static_cast<const __half*>(beta);
  uint8_t* q = static_cast<uint8_t*>(q_out);
  const int d = static_cast<int>(D);
  if (rows > 0) {
    if (int e = launch_ln_mode<kModeStats, WBK_FMT_E4M3>(xh, gh, bh, rows, d, eps, amax_ws, stats, nullptr, nullptr,
                                                          nullptr, s))
      return e;
  }
  // scale only (1.0); scale_out is left unwritten like an empty quantise
  if (rows == 0) return wbk_scale_from_amax(amax_ws, fmt, scale_inv, stream);
  // The quantise pass derives the scale from the amax itself.
  return fmt == WBK_FMT_E4M3
             ? launch_ln_mode<kModeQuant, WBK_FMT_E4M3>(xh, gh, bh, rows, d, eps, amax_ws, stats, scale_inv, q,
                                                         scale_out, s)
             : launch_ln_mode<kModeQuant, WBK_FMT_E5M2>(xh, gh, bh, rows, d, eps, amax_ws, stats, scale_inv, q,
                                                         scale_out, s);
}

}  // extern "C"
