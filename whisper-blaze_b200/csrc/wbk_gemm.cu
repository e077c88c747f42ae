// FP8 x FP8 -> FP32 (TMEM) -> FP16 per-tensor-scaled GEMM on B200 tcgen05.
//
//   out[M,N] = epilogue((A[M,K] . W[N,K]^T) * descale + bias ...)
//
// The reference has no working FP8 GEMM: its Hopper wgmma kernel
// (csrc/kernels/gemm_hopper.cu:179-269) is unbound, and BlazeLinear.forward
// (whisper_blaze/model.py:80-109) dequantises both operands and calls an fp16
// F.linear. This kernel computes what that path means — descale = a_scale *
// w_scale applied to an fp32 accumulator, then bias, then fp16 (the intent of
// gemm_hopper.cu:251-268) — natively on 5th-generation tensor cores:
//
//   * persistent grid, one CTA per SM, static round-robin over 128x256 tiles
//     (N-fastest so consecutive CTAs share the A row-block in L2);
//   * warp 0: TMA producer. A [128 x 128 B] and W [256 x 128 B] boxes, 128-byte
//     swizzle, into a 4-stage shared-memory ring (48 KB per stage);
//   * warp 1: TMEM owner + single-thread tcgen05.mma issuer
//     (kind::f8f6f4, M=128 N=256 K=32, fp32 accumulate), committing each stage
//     back to the producer and each finished tile to the epilogue;
//   * warps 2-9: epilogue. Two 256-column fp32 accumulators in TMEM (all 512
//     columns) so the epilogue of tile i overlaps the MMAs of tile i+1. Warp w
//     may only touch TMEM lanes 32*(w%4)..+31, so two warps share each lane
//     quarter and split the 256 columns in halves. Each drains 32-column
//     chunks with double-buffered tcgen05.ld, applies descale, bias, exact-erf
//     GELU or residual add (+ fp16 clamp), rounds to fp16, tracks max|out|,
//     and writes the chunk through a 64B-swizzled shared-memory staging
//     buffer with a TMA bulk-tensor store (coalesced, asynchronous, clipped at
//     the M/N edges by the hardware). Outputs whose row pitch is not a multiple
//     of 16 bytes (N % 8 != 0) are stored directly from registers instead.
//
// Every mbarrier wait is bounded (wall-clock limit via %globaltimer): a wait
// that runs out records WBK_ERR_DEVICE_TIMEOUT in a device word, raises a
// CTA-wide abort flag so the other roles stop, drains its in-flight work with
// bounded waits, releases TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>
#include <string>
#include <type_traits>
#include <vector>

#include "wbk_common.cuh"
#include "wbk_fp8_quant.cuh"
#include "wbk_sm100.cuh"

namespace wbk {

namespace {

constexpr int BM = 128;
constexpr int BK = 128;  // bytes of K per stage = fp8 elements = one 128-byte swizzle row
constexpr int UMMA_K = 32;
constexpr int NUM_ACC = 2;
constexpr int EPI_WARPS = 8;
constexpr int THREADS = 64 + EPI_WARPS * 32;  // 320
constexpr int CHUNK = 32;                     // columns per tcgen05.ld / per TMA store box
constexpr int STAGE_OUT_BYTES = 32 * CHUNK * 2;  // 32 rows x 32 fp16 = 2 KB

// Output tile width kBN (MMA N): 256 for large GEMMs; 128 / 64 give more tiles
// for short-M shapes (the decoder step's M = 64) so every SM streams weights.
// kPair: a cluster of two CTAs on one TPC computes a 256 x kBN tile with
// tcgen05 cta_group::2 MMAs; each CTA loads its own 128 A rows and half of the
// kBN weight rows, so per-SM operand traffic (L2 and shared memory) is a third
// lower than one CTA computing 128 x kBN.
template <int kBN, bool kPair = false>
struct Tile {
  static constexpr int B_ROWS = kPair ? kBN / 2 : kBN;  // weight rows this CTA loads per K block
  static constexpr int B_SUB_BYTES = B_ROWS * BK;       // 32 / 16 / 8 KB (16 KB per CTA in a pair)
  // K blocks per pipeline stage: one TMA load per operand and one full/empty
  // barrier round trip serve G K blocks, so the single producer and MMA
  // threads spend 1/G of the per-block issue cost (each barrier operation or
  // TMA issue costs ~30-60 ns of one thread's time).
  static constexpr int G = kBN == 64 ? 4 : 2;
  static constexpr int A_STAGE_BYTES = G * BM * BK;     // room for G 128-row A blocks
  static constexpr int B_STAGE_BYTES = G * B_SUB_BYTES;
  // Shared-memory ring depth: ~192 KB of operands in flight per SM whatever the shape.
  static constexpr int STAGES = (192 * 1024) / (A_STAGE_BYTES + B_STAGE_BYTES);
  static constexpr int TMEM_COLS = NUM_ACC * kBN;    // 512 / 256 / 128 (power of two >= 32)
  static constexpr int EPI_COLS = kBN / 2;           // columns per epilogue warp (two warps per lane quarter)
  static constexpr int ROWS = kPair ? 2 * BM : BM;   // output rows per (pair) tile
  static_assert(kBN == 64 || kBN == 128 || kBN == 256, "tile width");
  static_assert(!kPair || kBN == 256, "CTA pairs use 256-wide tiles");
};

enum : uint32_t {
  SITE_PRODUCER_EMPTY = 1,
  SITE_MMA_ACC_EMPTY = 2,
  SITE_MMA_FULL = 3,
  SITE_EPI_ACC_FULL = 4,
  SITE_DRAIN = 5,
  SITE_QUANT_SYNC = 6,
  SITE_EPI_RES = 7,
  SITE_SELFTEST = 15,
};

// Shared-memory scratch of the in-kernel activation quantise.
struct QuantScratch {
  uint32_t red[THREADS / 32];  // per-warp amax
  uint32_t amax;
  float scale, inv;
  int ok;
};

template <int kBN, bool kPair = false>
struct SharedStorage {
  uint8_t a[Tile<kBN, kPair>::STAGES][Tile<kBN, kPair>::A_STAGE_BYTES];  // 1024-byte aligned (swizzle atom)
  uint8_t b[Tile<kBN, kPair>::STAGES][Tile<kBN, kPair>::B_STAGE_BYTES];
  uint8_t out[EPI_WARPS][2][STAGE_OUT_BYTES];  // per-warp double-buffered store staging
  uint64_t full[Tile<kBN, kPair>::STAGES];
  uint64_t empty[Tile<kBN, kPair>::STAGES];
  uint64_t acc_full[NUM_ACC];
  uint64_t acc_empty[NUM_ACC];
  uint64_t res_full[EPI_WARPS][2];  // residual box landed in out[warp][buffer] (TMA residual path)
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  QuantScratch q;  // in-kernel activation quantise (short-M linear)
};
template <int kBN, bool kPair = false>
constexpr size_t smem_bytes() { return sizeof(SharedStorage<kBN, kPair>) + 1024; }
static_assert(smem_bytes<256>() <= 232448 && smem_bytes<128>() <= 232448 && smem_bytes<64>() <= 232448 &&
                  smem_bytes<256, true>() <= 232448,
              "shared memory budget");

struct Params {
  int M, N, K;
  int tiles_n, num_tiles, kblocks;
  float alpha;
  const float* a_scale;
  const float* w_scale;
  const __half* bias;
  const __half* residual;
  __half* out;
  uint32_t* out_amax;
  int out_pairs;  // direct-store path: rows 4-byte aligned, store fp16 pairs
  uint32_t a_box_bytes;  // bytes of one A K block (64 or 128 rows x 128 B); A blocks are this far apart in a stage
  int grouped;           // 1: one 3-D TMA load per operand per stage (K % 128 == 0); 0: G 2-D loads
  uint32_t idesc;
  uint64_t timeout_ns;
  // Split-K (64-wide tiles only): work item = (tile, K slice); num_items = num_tiles * splits.
  int splits;
  int num_items;
  float* ws_partials;     // [num_items][128 rows][64 cols] fp32
  uint32_t* ws_tickets;   // [num_tiles][EPI_WARPS] arrival counts, zero between calls
  // CTA pairs: items [0, full_items) are whole tiles; each tile past them is split
  // into 2^narrow_shift column pieces (items of kBN >> narrow_shift columns, MMA N
  // likewise), so a partial last round of whole tiles becomes a shorter round of
  // narrow items. The narrow items' weight boxes come from the tensor map slot the
  // kernel does not otherwise use (tmap_w when loads are grouped, else tmap_w3).
  int full_items;
  int narrow_shift;
};

// Pair item -> (tile, first column inside the tile, width in columns).
template <int kBN>
__device__ __forceinline__ void pair_item(const Params& p, int item, int& tile, int& col_off, int& width) {
  if (item < p.full_items) {
    tile = item;
    col_off = 0;
    width = kBN;
    return;
  }
  const int j = item - p.full_items;
  tile = p.full_items + (j >> p.narrow_shift);
  width = kBN >> p.narrow_shift;
  col_off = (j & ((1 << p.narrow_shift) - 1)) * width;
}

// Parameters of the in-kernel activation quantise (64-wide tiles, cooperative
// launch): A is quantised per tensor from a_f16 into a_q, which the TMA then
// reads as A. Only those kernels take the larger block (ptxas allocates the
// other kernels' registers differently when their parameter block grows).
struct QuantParams : Params {
  const __half* a_f16;    // [M, K] fp16, rows contiguous
  uint8_t* a_q;           // [M, K] fp8 codes (out)
  float* a_scale_out;     // the quantiser's scale (out, may be null)
  uint32_t* a_amax_out;   // the quantiser's amax bits (out, may be null)
  uint32_t* qsync;        // 4 workspace words: arrivals (amax), arrivals (codes), departures, amax; zero between calls
  int64_t a_vecs;         // M * K / 8 (16-byte vectors of A)
  float a_max_fp8;
  int a_e5m2;
};
template <bool kQuantA>
using KernelParams = typename std::conditional<kQuantA, QuantParams, Params>::type;

// K blocks [kb0, kb1) of split `split`, whole stages of g blocks (every split
// gets at least one stage when splits <= stages).
__device__ __forceinline__ void split_range(const Params& p, int g, int split, int& kb0, int& kb1) {
  if (p.splits == 1) {  // the common case, without integer division on the critical path
    kb0 = 0;
    kb1 = p.kblocks;
    return;
  }
  const int nst = (p.kblocks + g - 1) / g;  // < 2^24 stages and <= 16 splits: 32-bit products suffice
  kb0 = (split * nst / p.splits) * g;
  kb1 = ((split + 1) * nst / p.splits) * g;
  if (kb1 > p.kblocks) kb1 = p.kblocks;
}

// Grid-wide arrival for the cooperatively launched (all CTAs co-resident)
// in-kernel quantise, run by one thread per CTA after a __syncthreads: a
// release add counts the CTA in *count (release is cumulative, so it also
// publishes the CTA's global writes that the barrier ordered before it), then
// an acquire poll waits until all `expected` CTAs have arrived. Bounded: gives
// up after `timeout_ns` of wall clock, recording the error.
__device__ __noinline__ bool grid_arrive_wait(uint32_t* count, uint32_t expected, uint64_t timeout_ns) {
  asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(count) : "memory");
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 0; it < (1u << 30); ++it) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(count) : "memory");
    if (v >= expected) return true;
    if ((it & 15u) == 15u && globaltimer_ns() - t0 > timeout_ns) break;
  }
  record_device_error(WBK_ERR_DEVICE_TIMEOUT, SITE_QUANT_SYNC);
  return false;
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Generic-proxy global writes <-> async-proxy (TMA) reads of the same bytes.
__device__ __forceinline__ void fence_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// In-kernel per-tensor quantise of A (cooperative launch, all THREADS threads
// of every CTA): each CTA takes the amax of its slice of a_f16, the grid agrees
// on the tensor's amax through one bounded grid-wide arrival, each CTA writes
// its slice's codes to a_q (read back by TMA afterwards), and after a second
// arrival CTA 0 publishes the scale and amax bits. The last CTA through zeroes
// the sync words for the next call. Returns false (timeout recorded) if an
// arrival gave up; the result is the same in every thread of the CTA.
// The arrivals are led by thread kQuantLeader, not thread 0: once A's loads for
// the amax have landed (so they do not queue behind the weight stream), thread
// 0 runs `issue_weights` (the early weight loads) while the leader arrives.
constexpr int kQuantLeader = 96;
template <class IssueWeights>
__device__ __forceinline__ bool quantise_a_prologue(const QuantParams& p, QuantScratch& q, IssueWeights&& issue_weights) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t v0 = p.a_vecs * blockIdx.x / gridDim.x;
  const int64_t v1 = p.a_vecs * (blockIdx.x + 1) / gridDim.x;
  const uint4* src = reinterpret_cast<const uint4*>(p.a_f16);
  uint32_t m = 0;
  for (int64_t i = v0 + threadIdx.x; i < v1; i += THREADS) m = max(m, absmax8_bits(__ldcg(src + i)));
  m = warp_max_u32(m);
  if (lane == 0) q.red[warp] = m;
  __syncthreads();
  if (threadIdx.x == 0) issue_weights();
  if (threadIdx.x == kQuantLeader) {
    uint32_t mm = 0;
#pragma unroll
    for (int w = 0; w < THREADS / 32; ++w) mm = max(mm, q.red[w]);
    if (mm != 0u) atomicMax(p.qsync + 3, mm);
    const bool ok = grid_arrive_wait(p.qsync + 0, gridDim.x, p.timeout_ns);
    const uint32_t amax = ok ? ld_acquire_gpu(p.qsync + 3) : 0u;
    float sc, inv;
    scale_from_amax(amax, p.a_max_fp8, sc, inv);
    q.amax = amax;
    q.scale = sc;
    q.inv = inv;
    q.ok = ok ? 1 : 0;
  }
  __syncthreads();
  if (q.ok) {
    const float inv = q.inv, mx = p.a_max_fp8;
    uint2* dst = reinterpret_cast<uint2*>(p.a_q);
    for (int64_t i = v0 + threadIdx.x; i < v1; i += THREADS) {
      const uint4 v = __ldcg(src + i);
      dst[i] = p.a_e5m2 ? make_uint2(q8x4<WBK_FMT_E5M2>(v.x, v.y, inv, mx), q8x4<WBK_FMT_E5M2>(v.z, v.w, inv, mx))
                        : make_uint2(q8x4<WBK_FMT_E4M3>(v.x, v.y, inv, mx), q8x4<WBK_FMT_E4M3>(v.z, v.w, inv, mx));
    }
    fence_async_global();  // the codes are read back by TMA (async proxy), in other CTAs too
  }
  __syncthreads();
  if (threadIdx.x == kQuantLeader && q.ok) {
    const bool ok = grid_arrive_wait(p.qsync + 1, gridDim.x, p.timeout_ns);
    if (ok) {
      if (blockIdx.x == 0) {
        if (p.a_scale_out != nullptr) *p.a_scale_out = q.scale;
        if (p.a_amax_out != nullptr) *p.a_amax_out = q.amax;
      }
      // Every CTA has passed both arrivals once the last one leaves: nothing reads the words again.
      if (atomicAdd(p.qsync + 2, 1u) == gridDim.x - 1u) {
        p.qsync[0] = 0u;
        p.qsync[1] = 0u;
        p.qsync[3] = 0u;
        p.qsync[2] = 0u;
      }
    }
    q.ok = ok ? 1 : 0;
  }
  __syncthreads();
  return q.ok != 0;
}

// ----------------------------------------------------------------- epilogue

template <int kEpi>
__device__ __forceinline__ float epi_apply(float v) {
  if (kEpi == WBK_EPI_GELU) v = gelu_erf(v);
  return v;
}

__device__ __forceinline__ void add_halves8(float* v, const uint4& raw) {
  const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const float2 f = __half22float2(h[t]);
    v[2 * t] += f.x;
    v[2 * t + 1] += f.y;
  }
}

__host__ __device__ constexpr bool has_residual(int epi) { return epi == WBK_EPI_RESIDUAL || epi == WBK_EPI_RESIDUAL_CLAMP; }

// Pulls this thread's 128-column residual row segment of `tile` (256 B, two
// 128-byte lines) into L2 ahead of use.
template <int kBN, int kEpi>
__device__ __forceinline__ void prefetch_residual_l2(const Params& p, int tile, int tile_rows, int row_off, int quarter,
                                                     int col_half, int lane) {
  if (!has_residual(kEpi) || tile >= p.num_tiles) return;
  const int row = (tile / p.tiles_n) * tile_rows + row_off + quarter * 32 + lane;
  const int col = (tile % p.tiles_n) * kBN + col_half * Tile<kBN>::EPI_COLS;
  if (row >= p.M || col >= p.N) return;
  const __half* base = p.residual + static_cast<int64_t>(row) * p.N + col;
  asm volatile("prefetch.global.L2 [%0];" ::"l"(base));
  if (Tile<kBN>::EPI_COLS > 64 && col + 64 < p.N) asm volatile("prefetch.global.L2 [%0];" ::"l"(base + 64));
}

// Issues the residual loads of one full 32-column chunk of this thread's row
// (4 x 16 B) so they are in flight while the previous chunk is processed.
// Partial chunks and rows >= M are handled by the scalar path in epi_values.
template <int kEpi, bool kVec>
__device__ __forceinline__ void prefetch_residual(const Params& p, int row, int col0, uint4* r) {
  if (has_residual(kEpi) && kVec && row < p.M && col0 + 32 <= p.N) {
    const uint4* rv = reinterpret_cast<const uint4*>(p.residual + static_cast<int64_t>(row) * p.N + col0);
#pragma unroll
    for (int q = 0; q < 4; ++q) r[q] = __ldg(rv + q);
  }
}

// fp32 accumulators of one 32-column chunk of this thread's row -> epilogue
// values in fp32 (descale, bias, activation, residual, clamp). Columns >= N
// and rows >= M are never read from global memory.
// bias_pre: the chunk's 32 bias values already loaded into registers (nullptr: load them).
// res_all: `res` holds the whole chunk (a TMA box, zero past row M and column N)
// even when the chunk is partial.
template <int kEpi, bool kVec>
__device__ __forceinline__ void epi_values(const Params& p, const uint32_t* acc, const uint4* res, int row, int col0,
                                           float descale, float* v, const uint4* bias_pre = nullptr,
                                           bool res_all = false) {
  const int N = p.N;
  const bool full = kVec && (col0 + 32 <= N);
  if (p.bias != nullptr && full) {
    const uint4* bv = reinterpret_cast<const uint4*>(p.bias + col0);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 b = bias_pre != nullptr ? bias_pre[q] : __ldg(bv + q);
      const __half2* h = reinterpret_cast<const __half2*>(&b);
#pragma unroll
      for (int t = 0; t < 4; ++t) {  // fma(acc, descale, bias), two lanes per instruction
        const float2 r = f2_fma(make_float2(__uint_as_float(acc[8 * q + 2 * t]), __uint_as_float(acc[8 * q + 2 * t + 1])),
                                make_float2(descale, descale), __half22float2(h[t]));
        v[8 * q + 2 * t] = r.x;
        v[8 * q + 2 * t + 1] = r.y;
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(acc[j]) * descale;
    if (p.bias != nullptr) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) v[j] += __half2float(p.bias[col0 + j]);
    }
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = epi_apply<kEpi>(v[j]);
  if (has_residual(kEpi)) {
    if (row < p.M) {
      if (full || res_all) {
#pragma unroll
        for (int q = 0; q < 4; ++q) add_halves8(v + 8 * q, res[q]);
      } else {
        const __half* rrow = p.residual + static_cast<int64_t>(row) * N;
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (col0 + j < N) v[j] += __half2float(rrow[col0 + j]);
      }
    }
    if (kEpi == WBK_EPI_RESIDUAL_CLAMP) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = fminf(fmaxf(v[j], -64504.0f), 64504.0f);
    }
  }
}

// Rounds v to fp16 into 16 packed words.
__device__ __forceinline__ void pack_fp16(const float* v, uint32_t* w) {
#pragma unroll
  for (int t = 0; t < 16; ++t) {
    const __half2 h = __floats2half2_rn(v[2 * t], v[2 * t + 1]);
    w[t] = *reinterpret_cast<const uint32_t*>(&h);
  }
}

// max (of |v| with kAbs) over a full 32-column chunk as a depth-5 tree of fmaxf instead of a
// 32-long dependent chain; fmaxf ignores NaN and is associative on everything else, so the
// result equals the sequential maximum.
template <bool kAbs>
__device__ __forceinline__ float tree_max32(const float* v) {
  float t[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) t[j] = kAbs ? fmaxf(fabsf(v[2 * j]), fabsf(v[2 * j + 1])) : fmaxf(v[2 * j], v[2 * j + 1]);
#pragma unroll
  for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
    for (int j = 0; j < w; ++j) t[j] = fmaxf(t[2 * j], t[2 * j + 1]);
  return t[0];
}

// Running (signed) max of v over the valid columns (fmaxf ignores NaN).
__device__ __forceinline__ float max_valid(float m, const float* v, int valid_cols) {
  if (valid_cols >= 32) return fmaxf(m, tree_max32<false>(v));
#pragma unroll
  for (int j = 0; j < 32; ++j)
    if (j < valid_cols) m = fmaxf(m, v[j]);
  return m;
}

// Running max of |v| over the valid columns (fmaxf ignores NaN). Rounding to
// fp16 is monotone and symmetric, so fp16(max |v|) is max |fp16(v)|.
__device__ __forceinline__ float absmax_valid(float m, const float* v, int valid_cols) {
  if (valid_cols >= 32) return fmaxf(m, tree_max32<true>(v));
#pragma unroll
  for (int j = 0; j < 32; ++j)
    if (j < valid_cols) m = fmaxf(m, fabsf(v[j]));
  return m;
}

// ------------------------------------------------------------------- kernel

// The residual's tensor map, a kernel parameter only of the TMA-residual variants
// (last in the parameter block, so the other kernels' parameters are unchanged).
template <bool kOn>
struct ResMap {
  CUtensorMap map;
};
template <>
struct ResMap<false> {};

// kResTma: CTA-pair residual epilogues only; the residual arrives by TMA in the store staging buffers.
template <int kBN, int kEpi, bool kTmaStore, bool kPair, bool kQuantA, bool kResTma = false>
__global__ void __launch_bounds__(THREADS, 1)
fp8_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_w,
                const __grid_constant__ CUtensorMap tmap_out, const __grid_constant__ CUtensorMap tmap_a3,
                const __grid_constant__ CUtensorMap tmap_w3, const KernelParams<kQuantA> p,
                const __grid_constant__ ResMap<kResTma> res_map) {
  extern __shared__ uint8_t smem_raw[];
  SharedStorage<kBN, kPair>& s =
      *reinterpret_cast<SharedStorage<kBN, kPair>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  using TL = Tile<kBN, kPair>;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  volatile int* abort_flag = &s.abort_flag;
  // Tiles are 128 x kBN per CTA, or 256 x kBN per CTA pair (rank r owns rows 128r..).
  const uint32_t rank = kPair ? cluster_ctarank() : 0u;
  const int first_tile = kPair ? static_cast<int>(cluster_id_x()) : static_cast<int>(blockIdx.x);
  const int tile_stride = kPair ? static_cast<int>(num_clusters_x()) : static_cast<int>(gridDim.x);
  const int row_off = static_cast<int>(rank) * BM;

  if (threadIdx.x == 0) {
    for (int i = 0; i < TL::STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < NUM_ACC; ++i) {
      mbar_init(&s.acc_full[i], 1);
      mbar_init(&s.acc_empty[i], kPair ? 2 * EPI_WARPS : EPI_WARPS);  // one arrival per epilogue warp (of the pair)
    }
    for (int i = 0; i < EPI_WARPS; ++i) {
      mbar_init(&s.res_full[i][0], 1);
      mbar_init(&s.res_full[i][1], 1);
    }
    mbar_init(&s.drain, 1);
    s.abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    if (p.grouped) {
      prefetch_tmap(&tmap_a3);
      prefetch_tmap(&tmap_w3);
    } else {
      prefetch_tmap(&tmap_a);
      prefetch_tmap(&tmap_w);
    }
    if (kTmaStore) prefetch_tmap(&tmap_out);
    if constexpr (kResTma) prefetch_tmap(&res_map.map);
  }
  if (warp == 1) {
    if (kPair) {
      tmem_alloc_pair(&s.tmem_base, TL::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(&s.tmem_base, TL::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (kPair) cluster_sync();  // the leader's barriers are initialised before the peer signals them
  tc_fence_after();
  const uint32_t tmem_base = s.tmem_base;
  // Launched with programmatic stream serialization: everything above overlaps
  // the kernel that produces A / the scales; nothing below runs before it is done.
  // A following kernel launched the same way may start its own prologue on SMs
  // this grid leaves free (its wait still blocks until this grid has finished).
  griddep_launch_dependents();
  griddep_wait();

  // TMA loads of one single-CTA stage: the A and/or W boxes of K blocks [kb, kb + G).
  auto load_stage = [&](int stage, int kb, int m0, int n0, bool load_a, bool load_w) {
    if (p.grouped) {
      if (load_a) tma_load_3d(&tmap_a3, &s.full[stage], s.a[stage], 0, m0, kb);
      if (load_w) tma_load_3d(&tmap_w3, &s.full[stage], s.b[stage], 0, n0, kb);
    } else {
#pragma unroll
      for (int g = 0; g < TL::G; ++g) {
        if (load_a) tma_load_2d(&tmap_a, &s.full[stage], s.a[stage] + g * p.a_box_bytes, (kb + g) * BK, m0);
        if (load_w) tma_load_2d(&tmap_w, &s.full[stage], s.b[stage] + g * TL::B_SUB_BYTES, (kb + g) * BK, n0);
      }
    }
  };

  // In-kernel quantise of A (short-M linear). Every CTA takes the amax of its
  // slice of A; the W boxes of the first stages go out once those loads have
  // landed and stream in meanwhile. The grid agrees on the tensor's amax (one
  // bounded grid-wide arrival; the launch is cooperative, so all CTAs are
  // resident), each CTA writes its slice's codes, and after a second arrival
  // the pipeline below TMA-loads A from those codes as usual. The last CTA
  // through zeroes the sync words for the next call.
  int pre = 0;  // stages whose W half was issued ahead of the quantise
  bool run = true;
  if constexpr (kQuantA) {
    static_assert(!kPair, "the in-kernel quantise is for single-CTA tiles");
    run = quantise_a_prologue(p, s.q, [&]() {
      if (first_tile >= p.num_items) return;
      const int tile = first_tile / p.splits;
      int kb0, kb1;
      split_range(p, TL::G, first_tile - tile * p.splits, kb0, kb1);
      const int n0 = (tile % p.tiles_n) * kBN;
      for (int kb = kb0; kb < kb1 && pre < TL::STAGES; kb += TL::G, ++pre) {
        mbar_arrive_expect_tx(&s.full[pre], TL::G * (p.a_box_bytes + TL::B_SUB_BYTES));
        load_stage(pre, kb, 0, n0, false, true);
      }
    });
  }

  if constexpr (kQuantA) {
    if (!run && warp == 0 && lane == 0 && pre > 0) {
      // The quantise gave up (timeout recorded): complete and wait out the stages
      // whose W boxes are in flight (A's bytes may be stale, nothing uses them).
      const int tile = first_tile / p.splits;
      int kb0, kb1;
      split_range(p, TL::G, first_tile - tile * p.splits, kb0, kb1);
      for (int i = 0; i < pre; ++i) load_stage(i, kb0 + i * TL::G, 0, 0, true, false);
      for (int i = 0; i < pre; ++i) {
        int dummy = 0;
        mbar_wait(&s.full[i], 0, &dummy, 1000000ull, SITE_DRAIN);
      }
    }
  }
  if (!run) {
    // nothing else runs: straight to the teardown
  } else if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int n_st = 0;  // stages issued so far; the first `pre` have their W half in flight already
      if constexpr (kQuantA) fence_async_global();
      for (int item = first_tile; item < p.num_items && ok; item += tile_stride) {
        int tile, col_off = 0, width = kBN;
        if constexpr (kPair) pair_item<kBN>(p, item, tile, col_off, width);
        else tile = item / p.splits;
        int kb0, kb1;
        split_range(p, TL::G, item - tile * p.splits, kb0, kb1);
        const int m0 = (tile / p.tiles_n) * TL::ROWS + row_off;
        // each CTA of a pair loads half of the item's weight rows
        const int n0 = (tile % p.tiles_n) * kBN + col_off + static_cast<int>(rank) * (kPair ? width / 2 : kBN);
        const uint32_t b_sub = kPair ? static_cast<uint32_t>(width / 2) * BK : static_cast<uint32_t>(TL::B_SUB_BYTES);
        const bool narrow = kPair && width < kBN;
        for (int kb = kb0; kb < kb1; kb += TL::G) {
          if constexpr (kQuantA) {
            if (n_st++ < pre) {  // W issued ahead: only A is left
              load_stage(stage, kb, m0, n0, true, false);
              if (++stage == TL::STAGES) {
                stage = 0;
                phase ^= 1u;
              }
              continue;
            }
          }
          if (!mbar_wait(&s.empty[stage], phase ^ 1u, abort_flag, p.timeout_ns, SITE_PRODUCER_EMPTY)) {
            ok = false;
            break;
          }
          // A stage always receives G whole boxes per operand (blocks past K read as zeros).
          const uint32_t stage_bytes = TL::G * (p.a_box_bytes + b_sub);
          if (kPair) {
            // Both CTAs' loads complete on the leader's full barrier, which expects both halves.
            if (rank == 0) mbar_arrive_expect_tx(&s.full[stage], 2 * stage_bytes);
            const uint32_t full_leader = mapa_shared(&s.full[stage], 0);
            if (p.grouped) {
              tma_load_3d_pair(&tmap_a3, full_leader, s.a[stage], 0, m0, kb);
              tma_load_3d_pair(narrow ? &tmap_w : &tmap_w3, full_leader, s.b[stage], 0, n0, kb);
            } else {
#pragma unroll
              for (int g = 0; g < TL::G; ++g) {
                tma_load_2d_pair(&tmap_a, full_leader, s.a[stage] + g * p.a_box_bytes, (kb + g) * BK, m0);
                tma_load_2d_pair(narrow ? &tmap_w3 : &tmap_w, full_leader, s.b[stage] + g * b_sub, (kb + g) * BK, n0);
              }
            }
          } else {
            mbar_arrive_expect_tx(&s.full[stage], stage_bytes);
            load_stage(stage, kb, m0, n0, true, true);
          }
          if (++stage == TL::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (ok) {
        // Producer tail: wait until the MMA warp has released every stage, so
        // no tcgen05.commit arrival to this CTA's barriers is still in flight
        // when it exits.
        int st = stage;
        uint32_t ph = phase;
        for (int i = 0; i < TL::STAGES && ok; ++i) {
          ok = mbar_wait(&s.empty[st], ph ^ 1u, abort_flag, p.timeout_ns, SITE_PRODUCER_EMPTY);
          if (++st == TL::STAGES) {
            st = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok) {
        // Abort path (in the loop or in the tail): let the copies already issued
        // land before the CTA exits. (stage, phase) is the ring position after the
        // last fill, so stage i was last filled with parity phase if i < stage,
        // else phase ^ 1 (a stage never filled then waits on the parity before
        // its first phase, which reads as complete).
        for (int i = 0; i < TL::STAGES && (!kPair || rank == 0); ++i) {
          const uint32_t ph = (i < stage) ? phase : (phase ^ 1u);
          int dummy = 0;
          mbar_wait(&s.full[i], ph, &dummy, 1000000ull, SITE_DRAIN);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    if (lane == 0 && (!kPair || rank == 0)) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int item = first_tile; item < p.num_items && ok; item += tile_stride) {
        int kb0, kb1;
        split_range(p, TL::G, item % p.splits, kb0, kb1);
        // narrow pair items: MMA N = the item's width, its weight rows stacked per K block
        uint32_t idesc = p.idesc;
        uint32_t b_sub = TL::B_SUB_BYTES;
        if constexpr (kPair) {
          int tile, col_off, width;
          pair_item<kBN>(p, item, tile, col_off, width);
          idesc = (p.idesc & ~(0x3Fu << 17)) | (static_cast<uint32_t>(width >> 3) << 17);
          b_sub = static_cast<uint32_t>(width / 2) * BK;
        }
        if (!mbar_wait(&s.acc_empty[acc], acc_phase ^ 1u, abort_flag, p.timeout_ns, SITE_MMA_ACC_EMPTY)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kBN);
        for (int kbs = kb0; kbs < kb1; kbs += TL::G) {
          if (!mbar_wait(&s.full[stage], phase, abort_flag, p.timeout_ns, SITE_MMA_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int g = 0; g < TL::G; ++g) {
            const int kb = kbs + g;
            if (kb >= kb1) break;
            const uint64_t adesc = make_sw128_desc(s.a[stage] + g * p.a_box_bytes);
            const uint64_t bdesc = make_sw128_desc(s.b[stage] + g * b_sub);
#pragma unroll
            for (int k = 0; k < BK / UMMA_K; ++k) {
              // Advance the start address by k*32 bytes inside the 128-byte swizzle row.
              const uint64_t koff = static_cast<uint64_t>((k * UMMA_K) >> 4);
              if (kPair)
                umma_f8f6f4_pair(d_tmem, adesc + koff, bdesc + koff, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
              else
                umma_f8f6f4(d_tmem, adesc + koff, bdesc + koff, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
            }
          }
          // frees this smem stage (in both CTAs of a pair) once its MMAs retire
          if (kPair) umma_commit_pair_mc(&s.empty[stage], 0x3);
          else umma_commit(&s.empty[stage]);
          if (++stage == TL::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        // accumulator ready for the epilogue (of both CTAs of a pair)
        if (kPair) umma_commit_pair_mc(&s.acc_full[acc], 0x3);
        else umma_commit(&s.acc_full[acc]);
        if (++acc == NUM_ACC) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok) {
        // Abort path: wait for every MMA this thread issued before TMEM is freed.
        if (kPair) umma_commit_pair(&s.drain);
        else umma_commit(&s.drain);
        int dummy = 0;
        mbar_wait(&s.drain, 0, &dummy, 1000000ull, SITE_DRAIN);
      }
    }
  } else {
    // --------------------------------------------------------- epilogue
    const int ew = warp - 2;             // 0..7
    const int quarter = warp & 3;        // TMEM lanes this warp may access: 32*quarter ..
    const int col_half = ew >> 2;        // which 128 of the 256 accumulator columns
    const float a_sc = kQuantA ? s.q.scale : (p.a_scale ? __ldg(p.a_scale) : 1.0f);
    const float descale = p.alpha * a_sc * (p.w_scale ? __ldg(p.w_scale) : 1.0f);
    constexpr bool kSignedMax = (kEpi == WBK_EPI_BIAS_MAXKEY);
    float amax = kSignedMax ? -INFINITY : 0.0f;  // max |out|, or max out for the key epilogue
    int acc = 0;
    uint32_t acc_phase = 0;
    int sbuf = 0;  // staging buffer toggle (kTmaStore)
    // CTA-pair residual epilogues (kResTma): each chunk's [32 rows x 32 columns]
    // residual box is loaded by TMA, one chunk ahead, into the staging buffer its
    // output is later stored from (same 64-byte swizzle), and the output overwrites
    // it in place. One TMA load per 2 KB box replaces 128 per-thread 16-byte loads
    // that each touch 32 rows.
    static_assert(!kResTma || (kPair && kTmaStore && has_residual(kEpi)), "TMA residual: CTA-pair residual epilogues");
    constexpr bool res_tma = kResTma;
    uint32_t res_phase = 0u;    // parity of res_full[ew][b], bit b
    uint32_t res_pending = 0u;  // buffers whose residual load has not been waited for
    bool res_ok = true;
    auto issue_res = [&](int b, int col0, int r0) {
      // After a failed wait no further load is issued: a buffer may still have one in
      // flight, and a second arrival on its barrier's pending phase is not allowed.
      if (!res_ok) return;
      if constexpr (kResTma) {
        if (lane == 0) {
          bulk_wait_read<0>();  // this warp's stores have finished reading their staging buffers
          mbar_arrive_expect_tx(&s.res_full[ew][b], STAGE_OUT_BYTES);
          tma_load_2d(&res_map.map, &s.res_full[ew][b], &s.out[ew][b][0], col0, r0);
        }
      }
      res_pending |= 1u << b;
    };
    prefetch_residual_l2<kBN, kEpi>(p, first_tile / p.splits, TL::ROWS, row_off, quarter, col_half, lane);
    for (int item = first_tile; item < p.num_items; item += tile_stride) {
      int tile, col_off = 0, epi_cols = TL::EPI_COLS;  // this warp's columns of the item
      if constexpr (kPair) {
        int width;
        pair_item<kBN>(p, item, tile, col_off, width);
        epi_cols = width / 2;
      } else {
        tile = item / p.splits;
      }
      if (!kPair || item + tile_stride < p.full_items)
        prefetch_residual_l2<kBN, kEpi>(p, (item + tile_stride) / p.splits, TL::ROWS, row_off, quarter, col_half,
                                        lane);  // next tile
      const int m0 = (tile / p.tiles_n) * TL::ROWS + row_off;
      const int n0 = (tile % p.tiles_n) * kBN + col_off + col_half * epi_cols;
      const int row0 = m0 + quarter * 32;
      const int row = row0 + lane;
      uint4 resa[4], resb[4];
      if (res_tma) {
        if (n0 < p.N) issue_res(sbuf, n0, row0);  // overlaps the tile's MMAs
      } else {
        prefetch_residual<kEpi, kTmaStore>(p, row, n0, resa);  // overlaps the tile's MMAs
      }
      // 64-wide tiles (one 32-column chunk per warp): the bias is loaded before the
      // accumulator wait too, off the short-M GEMMs' critical path.
      uint4 bpre[4];
      const bool bias_early = kBN == 64 && kTmaStore && p.bias != nullptr && n0 + CHUNK <= p.N;
      if (bias_early) {
#pragma unroll
        for (int q = 0; q < 4; ++q) bpre[q] = __ldg(reinterpret_cast<const uint4*>(p.bias + n0) + q);
      }
      if (!mbar_wait(&s.acc_full[acc], acc_phase, abort_flag, p.timeout_ns, SITE_EPI_ACC_FULL)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             static_cast<uint32_t>(acc * kBN + col_half * epi_cols);
      const int nchunks = min(epi_cols / CHUNK, (p.N - n0 + CHUNK - 1) / CHUNK);  // warp-uniform, may be <= 0
      auto process = [&](const uint32_t* regs, const uint4* res, int c, const uint4* bias_reg) {
        const int col0 = n0 + c * CHUNK;
        uint4 rs[4];
        if constexpr (res_tma) {
          const uint8_t* rbuf = &s.out[ew][0][0] + sbuf * STAGE_OUT_BYTES;
          const bool landed =
              res_ok && mbar_wait(&s.res_full[ew][sbuf], (res_phase >> sbuf) & 1u, abort_flag, p.timeout_ns, SITE_EPI_RES);
          if (__all_sync(0xFFFFFFFFu, landed)) {  // warp-uniform phase and pending state
            res_phase ^= 1u << sbuf;
            res_pending &= ~(1u << sbuf);
          } else {
            res_ok = false;  // the tile loop ends after this tile; pending loads are drained at exit
          }
#pragma unroll
          for (int q = 0; q < 4; ++q)
            rs[q] = *reinterpret_cast<const uint4*>(rbuf + lane * 64 + (q ^ ((lane >> 1) & 3)) * 16);
        }
        float v[32];
        epi_values<kEpi, kTmaStore>(p, regs, res_tma ? rs : res, row, col0, descale, v,
                                    bias_reg != nullptr ? bias_reg : ((bias_early && c == 0) ? bpre : nullptr),
                                    res_tma);
        const int valid_cols = (row < p.M) ? min(CHUNK, p.N - col0) : 0;
        if (kSignedMax || p.out_amax != nullptr)  // the running max only when an amax is asked for
          amax = kSignedMax ? max_valid(amax, v, valid_cols) : absmax_valid(amax, v, valid_cols);
        uint32_t w[16];
        pack_fp16(v, w);
        if (kTmaStore) {
          // Stage [32 rows x 64 B] with the 64-byte swizzle (16-byte chunk index
          // XOR (row/2)%4), then one lane stores the box with TMA. With the TMA
          // residual each lane overwrites only the 64 bytes it has just read, and
          // the buffer was free before its residual load was issued.
          uint8_t* buf = &s.out[ew][0][0] + sbuf * STAGE_OUT_BYTES;
          if (!res_tma) {
            if (lane == 0) bulk_wait_read<1>();  // the store that last read `buf` is done
            __syncwarp();
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int chunk16 = q ^ ((lane >> 1) & 3);
            *reinterpret_cast<uint4*>(buf + lane * 64 + chunk16 * 16) =
                make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
          }
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmap_out, buf, col0, row0);
            bulk_commit();
          }
          sbuf ^= 1;
        } else if (row < p.M) {
          __half* orow = p.out + static_cast<int64_t>(row) * p.N + col0;
          if (p.out_pairs) {  // even N, 4-byte aligned rows: store fp16 pairs
            uint32_t* o32 = reinterpret_cast<uint32_t*>(orow);
#pragma unroll
            for (int t = 0; t < 16; ++t)
              if (2 * t + 1 < valid_cols) o32[t] = w[t];
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < valid_cols)
                orow[j] = __ushort_as_half(static_cast<unsigned short>((w[j >> 1] >> ((j & 1) * 16)) & 0xFFFFu));
          }
        }
      };
      // Split-K: park this warp's fp32 partial (rows of its lane quarter, its
      // columns) in the workspace; the warp whose ticket completes the tile's
      // count sums every split's partial in split order (bit-deterministic) and
      // runs the epilogue. Returns false when this warp has nothing to store.
      auto split_reduce = [&](const uint32_t* regs, int c, uint32_t* sum) -> bool {
        const int trow = quarter * 32 + lane;  // row inside the 128-row tile
        const int tcol = col_half * TL::EPI_COLS + c * CHUNK;
        const size_t stride_item = static_cast<size_t>(TL::ROWS) * kBN;
        if (row < p.M) {
          float4* dst = reinterpret_cast<float4*>(p.ws_partials + static_cast<size_t>(item) * stride_item +
                                                  static_cast<size_t>(trow) * kBN + tcol);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            __stcg(dst + q, make_float4(__uint_as_float(regs[4 * q]), __uint_as_float(regs[4 * q + 1]),
                                        __uint_as_float(regs[4 * q + 2]), __uint_as_float(regs[4 * q + 3])));
        }
        __threadfence();
        __syncwarp();
        uint32_t last = 0;
        if (lane == 0) {
          constexpr int kChunks = TL::EPI_COLS / CHUNK;
          uint32_t* t = p.ws_tickets + (static_cast<size_t>(tile) * EPI_WARPS + quarter * 2 + col_half) * kChunks + c;
          last = atomicAdd(t, 1u) == static_cast<uint32_t>(p.splits - 1) ? 1u : 0u;
          if (last) *t = 0u;  // every split has arrived: leave the ticket zero for the next call
        }
        last = __shfl_sync(0xFFFFFFFFu, last, 0);
        if (!last) return false;
        __threadfence();
#pragma unroll
        for (int j = 0; j < 32; ++j) sum[j] = 0u;
        if (row < p.M) {
          float f[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) f[j] = 0.0f;
          // Slices are added in order 0, 1, 2, ...; the loads of two slices are in
          // flight together (more would spill the epilogue's registers).
          const float* base = p.ws_partials + static_cast<size_t>(tile) * p.splits * stride_item +
                              static_cast<size_t>(trow) * kBN + tcol;
          for (int sp = 0; sp < p.splits; sp += 2) {
            float4 v4[2][8];
#pragma unroll
            for (int u = 0; u < 2; ++u)
              if (sp + u < p.splits) {
                const float4* src = reinterpret_cast<const float4*>(base + static_cast<size_t>(sp + u) * stride_item);
#pragma unroll
                for (int q = 0; q < 8; ++q) v4[u][q] = __ldcg(src + q);
              }
#pragma unroll
            for (int u = 0; u < 2; ++u)
              if (sp + u < p.splits) {
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                  f[4 * q] += v4[u][q].x;
                  f[4 * q + 1] += v4[u][q].y;
                  f[4 * q + 2] += v4[u][q].z;
                  f[4 * q + 3] += v4[u][q].w;
                }
              }
          }
#pragma unroll
          for (int j = 0; j < 32; ++j) sum[j] = __float_as_uint(f[j]);
        }
        return true;
      };
      auto finish = [&](const uint32_t* regs, const uint4* res, int c, const uint4* bias_reg) {
        if constexpr (kBN == 64 && !kPair) {  // split-K exists only for the 64-wide (short-M) tiles
          if (p.splits > 1) {
            uint32_t sum[32];
            if (split_reduce(regs, c, sum)) process(sum, res, c, nullptr);
            return;
          }
        }
        process(regs, res, c, bias_reg);
      };
      // Double-buffered drain: the TMEM load and the residual loads of chunk c+1
      // are in flight while chunk c is processed.
      uint32_t ra[32], rb[32];
      if (nchunks > 0) {
        tmem_ld_32x32b_x32(taddr, ra);
        tmem_ld_wait(ra);
      }
#pragma unroll 1
      for (int c = 0; c < nchunks; c += 2) {
        const bool more1 = c + 1 < nchunks, more2 = c + 2 < nchunks;
        // process() advances sbuf, so sbuf ^ 1 is always the buffer of the chunk after the current one.
        if (more1) {
          tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>((c + 1) * CHUNK), rb);
          if (res_tma) issue_res(sbuf ^ 1, n0 + (c + 1) * CHUNK, row0);
          else prefetch_residual<kEpi, kTmaStore>(p, row, n0 + (c + 1) * CHUNK, resb);
        }
        finish(ra, resa, c, nullptr);
        if (more1) {
          tmem_ld_wait(rb);
          if (more2) {
            tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>((c + 2) * CHUNK), ra);
            if (res_tma) issue_res(sbuf ^ 1, n0 + (c + 2) * CHUNK, row0);
            else prefetch_residual<kEpi, kTmaStore>(p, row, n0 + (c + 2) * CHUNK, resa);
          }
          finish(rb, resb, c + 1, nullptr);
          if (more2) tmem_ld_wait(ra);
        }
      }
      if (!res_ok) break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (kPair && rank != 0) mbar_arrive_remote(mapa_shared(&s.acc_empty[acc], 0));  // the leader's barrier
        else mbar_arrive(&s.acc_empty[acc]);
      }
      if (++acc == NUM_ACC) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    // Abort path: a residual load that was never waited for may still be writing
    // shared memory; wait for it (bounded) before the CTA can exit.
    if (res_tma && res_pending != 0u) {
      int no_abort = 0;
      for (int b = 0; b < 2; ++b)
        if (res_pending & (1u << b))
          mbar_wait(&s.res_full[ew][b], (res_phase >> b) & 1u, &no_abort, 1000000ull, SITE_DRAIN);
    }
    // The staging buffers must have been read before the CTA exits; the global
    // writes themselves complete with the grid.
    if (kTmaStore && lane == 0) bulk_wait_read<0>();
    if (p.out_amax != nullptr) {
      const uint32_t h = __half_as_ushort(__float2half_rn(amax));
      const uint32_t bits = warp_max_u32(kSignedMax ? f16_order_key(h) : h);
      if (lane == 0 && bits != 0u) atomicMax(p.out_amax, bits);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (kPair) cluster_sync();  // neither CTA leaves while its pair may still touch its shared memory or TMEM
  if (warp == 1) {
    tc_fence_after();
    if (kPair) tmem_dealloc_pair(tmem_base, TL::TMEM_COLS);
    else tmem_dealloc(tmem_base, TL::TMEM_COLS);
  }
}

// ------------------------------------------------------ skinny (M <= 64) GEMM
//
// Decoder-step shapes (M <= 64 rows, K <= 1536) stream a large weight through
// every SM for a small A. This kernel keeps A resident in shared memory, loaded
// once per CTA (two K blocks per box and barrier), and gives the rest of shared
// memory to a weight-only ring, so more of the weight stream is in flight and
// no CTA re-reads A per tile. Tiles are 64 (or 128) output columns x all rows;
// the MMA is M = 128, so TMEM lanes 64..127 hold rows that do not exist: A's K
// blocks sit 8 KB (64 rows) apart and the MMA's rows 64..127 of block j read
// block j+1 (or, for the last block, 8 KB of slack), and those rows are never
// stored. Only the epilogue warps of lane quarters 0 and 1 (rows 0..63) work.
// Same per-tile MMA sequence as fp8_gemm_kernel, so the outputs are identical.
constexpr int kSkMaxStages = 12;
constexpr int kSkRows = 64;                          // A rows held (M <= 64)
constexpr int kSkABlock = kSkRows * BK;              // 8 KB per K block
constexpr int kSkASlack = (BM - kSkRows) * BK;       // the MMA's last-block overrun
constexpr int kSkEpiWarps = 4;                       // warps of lane quarters 0, 1 x two column halves
constexpr int kSkMaxKBlocks = 12;                    // K <= 1536
constexpr int kSkStageOut = 2 * STAGE_OUT_BYTES;     // per active epilogue warp, double-buffered

// kG: K blocks per weight stage. 2 in general; 5 when K is a multiple of 640
// (K = 1280: 40 KB boxes; a TMA probe streamed 40 KB boxes ~5 % faster than 16 KB ones).
template <int kBN, int kG = 2>
struct Skinny {
  static constexpr int G = kG;
  static constexpr int B_STAGE = G * kBN * BK;       // 16 / 40 KB (64-wide), 32 KB (128-wide)
  static constexpr int EPI_COLS = kBN / 2;           // columns per epilogue warp
  static constexpr int TMEM_COLS = NUM_ACC * kBN;
};

struct SkinnyHeader {  // at the (1024-aligned) start of shared memory
  uint64_t full[kSkMaxStages];
  uint64_t empty[kSkMaxStages];
  uint64_t a_full[kSkMaxKBlocks / 2];  // one per pair of A's K blocks
  uint64_t acc_full[NUM_ACC];
  uint64_t acc_empty[NUM_ACC];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  QuantScratch q;
};
constexpr int kSkHeaderBytes = 1024;
static_assert(sizeof(SkinnyHeader) <= kSkHeaderBytes, "skinny header");

struct SkinnyParams : QuantParams {
  int stages;           // weight ring depth
  uint32_t a_region;    // bytes of the resident A region (K blocks x 8 KB + slack), 1024-multiple
  int a_grouped;        // 1: one 3-D box brings all of A
  // Work items: items [0, full_items) are whole kBN-wide tiles; the columns past
  // them are split into kBN/2-wide items, so a last partial round of whole tiles
  // becomes one round of half tiles on up to twice as many CTAs.
  int full_items;
  uint32_t idesc_half;  // instruction descriptor of the kBN/2-wide MMA
};

// Dynamic shared memory of a skinny launch.
__host__ __device__ constexpr size_t skinny_smem(uint32_t a_region, int stages, int b_stage) {
  return 1024 + kSkHeaderBytes + a_region + static_cast<size_t>(stages) * b_stage + kSkEpiWarps * kSkStageOut;
}

template <int kBN, int kEpi, bool kTmaStore, bool kQuantA, int kG>
__global__ void __launch_bounds__(THREADS, 1)
fp8_skinny_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_w,
                  const __grid_constant__ CUtensorMap tmap_out, const __grid_constant__ CUtensorMap tmap_a3,
                  const __grid_constant__ CUtensorMap tmap_w3, const __grid_constant__ CUtensorMap tmap_wh,
                  const SkinnyParams p) {
  using SK = Skinny<kBN, kG>;
  constexpr int kHalf = kBN / 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  SkinnyHeader& h = *reinterpret_cast<SkinnyHeader*>(base);
  uint8_t* a_smem = base + kSkHeaderBytes;
  uint8_t* b_smem = a_smem + p.a_region;
  uint8_t* out_smem = b_smem + static_cast<size_t>(p.stages) * SK::B_STAGE;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  volatile int* abort_flag = &h.abort_flag;
  const int stages = p.stages;

  if (threadIdx.x == 0) {
    for (int i = 0; i < stages; ++i) {
      mbar_init(&h.full[i], 1);
      mbar_init(&h.empty[i], 1);
    }
    for (int i = 0; i < kSkMaxKBlocks / 2; ++i) mbar_init(&h.a_full[i], 1);
    for (int i = 0; i < NUM_ACC; ++i) {
      mbar_init(&h.acc_full[i], 1);
      mbar_init(&h.acc_empty[i], kSkEpiWarps);
    }
    mbar_init(&h.drain, 1);
    h.abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    if (p.a_grouped) prefetch_tmap(&tmap_a3);
    else prefetch_tmap(&tmap_a);
    if (p.grouped) prefetch_tmap(&tmap_w3);
    else prefetch_tmap(&tmap_w);
    if (kTmaStore) prefetch_tmap(&tmap_out);
  }
  if (warp == 1) {
    tmem_alloc(&h.tmem_base, SK::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = h.tmem_base;
  griddep_launch_dependents();  // as in fp8_gemm_kernel
  griddep_wait();

  // Item t: first column and whether it is a half-width tile.
  auto item_n0 = [&](int t) { return t < p.full_items ? t * kBN : p.full_items * kBN + (t - p.full_items) * kHalf; };
  // W boxes of K blocks [kb, kb + G) of the item at column n0 into ring stage `st`
  // (kBN rows, or kBN/2 rows for a half item, stacked per K block).
  auto load_w = [&](int st, int kb, int n0, bool half) {
    uint8_t* dst = b_smem + static_cast<size_t>(st) * SK::B_STAGE;
    mbar_arrive_expect_tx(&h.full[st], half ? SK::B_STAGE / 2 : SK::B_STAGE);
    if (p.grouped) {
      tma_load_3d(half ? &tmap_wh : &tmap_w3, &h.full[st], dst, 0, n0, kb);
    } else {
      const int rows = half ? kHalf : kBN;
#pragma unroll
      for (int g = 0; g < SK::G; ++g)
        tma_load_2d(half ? &tmap_wh : &tmap_w, &h.full[st], dst + g * rows * BK, (kb + g) * BK, n0);
    }
  };
  // All of A (every K block, 64-row boxes) into the resident region, two K blocks
  // per box and barrier, so the first MMAs wait for their own blocks only.
  auto load_a = [&]() {
    for (int j = 0; j * 2 < p.kblocks; ++j) {
      const int nb = min(2, p.kblocks - 2 * j);
      mbar_arrive_expect_tx(&h.a_full[j], static_cast<uint32_t>(p.a_grouped ? 2 : nb) * kSkABlock);
      if (p.a_grouped) {
        tma_load_3d(&tmap_a3, &h.a_full[j], a_smem + 2 * j * kSkABlock, 0, 0, 2 * j);
      } else {
        for (int kb = 2 * j; kb < 2 * j + nb; ++kb)
          tma_load_2d(&tmap_a, &h.a_full[j], a_smem + kb * kSkABlock, kb * BK, 0);
      }
    }
  };

  int pre = 0;  // ring stages whose weight boxes went out before the in-kernel quantise
  bool run = true;
  if constexpr (kQuantA) {
    run = quantise_a_prologue(p, h.q, [&]() {
      for (int t = blockIdx.x, kb = 0; t < p.num_tiles && pre < stages; ++pre) {
        load_w(pre, kb, item_n0(t), t >= p.full_items);
        kb += SK::G;
        if (kb >= p.kblocks) {
          kb = 0;
          t += gridDim.x;
        }
      }
    });
    if (!run && warp == 0 && lane == 0) {
      // complete the ring stages in flight before leaving (A's bytes are not used)
      for (int i = 0; i < pre; ++i) {
        int dummy = 0;
        mbar_wait(&h.full[i], 0, &dummy, 1000000ull, SITE_DRAIN);
      }
    }
  }

  if (!run) {
    // straight to the teardown
  } else if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      if constexpr (kQuantA) fence_async_global();  // A's codes were written by the generic proxy
      load_a();
      int st = 0;
      uint32_t phase = 0;
      int n_st = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        const int n0 = item_n0(tile);
        const bool half = tile >= p.full_items;
        for (int kb = 0; kb < p.kblocks; kb += SK::G) {
          if (!(kQuantA && n_st < pre)) {
            if (!mbar_wait(&h.empty[st], phase ^ 1u, abort_flag, p.timeout_ns, SITE_PRODUCER_EMPTY)) {
              ok = false;
              break;
            }
            load_w(st, kb, n0, half);
          }
          ++n_st;
          if (++st == stages) {
            st = 0;
            phase ^= 1u;
          }
        }
      }
      int dummy = 0;
      if (ok) {
        int st2 = st;
        uint32_t ph2 = phase;
        for (int i = 0; i < stages && ok; ++i) {  // every stage released: no commit arrival still in flight
          ok = mbar_wait(&h.empty[st2], ph2 ^ 1u, abort_flag, p.timeout_ns, SITE_PRODUCER_EMPTY);
          if (++st2 == stages) {
            st2 = 0;
            ph2 ^= 1u;
          }
        }
      }
      if (!ok) {
        // (st, phase) is the ring position after the last fill (the tail above did not move it)
        for (int i = 0; i < stages; ++i) {  // let the copies already issued land
          const uint32_t ph = (i < st) ? phase : (phase ^ 1u);
          mbar_wait(&h.full[i], ph, &dummy, 1000000ull, SITE_DRAIN);
        }
      }
      for (int j = 0; j * 2 < p.kblocks; ++j) mbar_wait(&h.a_full[j], 0, &dummy, ok ? p.timeout_ns : 1000000ull, SITE_DRAIN);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int st = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool a_ready = false;  // every A block landed (checked during the first tile)
      int a_next = 0;        // next pair of A blocks whose barrier is still to be waited on
      for (int tile = blockIdx.x; tile < p.num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(&h.acc_empty[acc], acc_phase ^ 1u, abort_flag, p.timeout_ns, SITE_MMA_ACC_EMPTY)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const bool half = tile >= p.full_items;
        const uint32_t idesc = half ? p.idesc_half : p.idesc;
        const int b_rows = half ? kHalf : kBN;
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kBN);
        for (int kbs = 0; kbs < p.kblocks; kbs += SK::G) {
          if (!mbar_wait(&h.full[st], phase, abort_flag, p.timeout_ns, SITE_MMA_FULL)) {
            ok = false;
            break;
          }
          if (!a_ready) {  // the A pairs this stage's K blocks need
            const int jlast = (min(kbs + SK::G, p.kblocks) - 1) >> 1;
            for (; a_next <= jlast && ok; ++a_next)
              ok = mbar_wait(&h.a_full[a_next], 0, abort_flag, p.timeout_ns, SITE_MMA_FULL);
            if (!ok) break;
            a_ready = 2 * a_next >= p.kblocks;
          }
          tc_fence_after();
          const uint8_t* bst = b_smem + static_cast<size_t>(st) * SK::B_STAGE;
#pragma unroll
          for (int g = 0; g < SK::G; ++g) {
            const int kb = kbs + g;
            if (kb >= p.kblocks) break;
            const uint64_t adesc = make_sw128_desc(a_smem + kb * kSkABlock);
            const uint64_t bdesc = make_sw128_desc(bst + g * b_rows * BK);
#pragma unroll
            for (int k = 0; k < BK / UMMA_K; ++k) {
              const uint64_t koff = static_cast<uint64_t>((k * UMMA_K) >> 4);
              umma_f8f6f4(d_tmem, adesc + koff, bdesc + koff, idesc, (kb > 0 || k > 0) ? 1u : 0u);
            }
          }
          umma_commit(&h.empty[st]);
          if (++st == stages) {
            st = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&h.acc_full[acc]);
        if (++acc == NUM_ACC) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok) {
        umma_commit(&h.drain);
        int dummy = 0;
        mbar_wait(&h.drain, 0, &dummy, 1000000ull, SITE_DRAIN);
      }
    }
  } else if ((warp & 3) < 2) {
    // --------------------------------------------------------- epilogue
    const int quarter = warp & 3;                   // 0 or 1: rows 32*quarter ..
    const int col_half = (warp - 2) >> 2;           // warps 4, 5: columns 0..; warps 8, 9: the second half
    const int ew = col_half * 2 + quarter;          // 0..3
    const float a_sc = kQuantA ? h.q.scale : (p.a_scale ? __ldg(p.a_scale) : 1.0f);
    const float descale = p.alpha * a_sc * (p.w_scale ? __ldg(p.w_scale) : 1.0f);
    constexpr bool kSignedMax = (kEpi == WBK_EPI_BIAS_MAXKEY);
    float amax = kSignedMax ? -INFINITY : 0.0f;
    int acc = 0;
    uint32_t acc_phase = 0;
    int sbuf = 0;
    const int row0 = quarter * 32;
    const int row = row0 + lane;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
      const int item0 = item_n0(tile);
      const int item_end = min(p.N, item0 + (tile >= p.full_items ? kHalf : kBN));
      const int n0 = item0 + col_half * SK::EPI_COLS;
      uint4 resa[4], resb[4];
      prefetch_residual<kEpi, kTmaStore>(p, row, n0, resa);
      if (!mbar_wait(&h.acc_full[acc], acc_phase, abort_flag, p.timeout_ns, SITE_EPI_ACC_FULL)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             static_cast<uint32_t>(acc * kBN + col_half * SK::EPI_COLS);
      const int nchunks = min(SK::EPI_COLS / CHUNK, (item_end - n0 + CHUNK - 1) / CHUNK);  // warp-uniform, may be <= 0
      auto process = [&](const uint32_t* regs, const uint4* res, int c) {
        const int col0 = n0 + c * CHUNK;
        float v[32];
        epi_values<kEpi, kTmaStore>(p, regs, res, row, col0, descale, v);
        const int valid_cols = (row < p.M) ? min(CHUNK, p.N - col0) : 0;
        if (kSignedMax || p.out_amax != nullptr)  // the running max only when an amax is asked for
          amax = kSignedMax ? max_valid(amax, v, valid_cols) : absmax_valid(amax, v, valid_cols);
        uint32_t w[16];
        pack_fp16(v, w);
        if (kTmaStore) {
          uint8_t* buf = out_smem + ew * kSkStageOut + sbuf * STAGE_OUT_BYTES;
          if (lane == 0) bulk_wait_read<1>();
          __syncwarp();
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int chunk16 = q ^ ((lane >> 1) & 3);
            *reinterpret_cast<uint4*>(buf + lane * 64 + chunk16 * 16) =
                make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
          }
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmap_out, buf, col0, row0);
            bulk_commit();
          }
          sbuf ^= 1;
        } else if (row < p.M) {
          __half* orow = p.out + static_cast<int64_t>(row) * p.N + col0;
          if (p.out_pairs) {
            uint32_t* o32 = reinterpret_cast<uint32_t*>(orow);
#pragma unroll
            for (int t = 0; t < 16; ++t)
              if (2 * t + 1 < valid_cols) o32[t] = w[t];
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < valid_cols)
                orow[j] = __ushort_as_half(static_cast<unsigned short>((w[j >> 1] >> ((j & 1) * 16)) & 0xFFFFu));
          }
        }
      };
      uint32_t ra[32], rb[32];
      if (nchunks > 0) {
        tmem_ld_32x32b_x32(taddr, ra);
        tmem_ld_wait(ra);
      }
#pragma unroll 1
      for (int c = 0; c < nchunks; c += 2) {
        const bool more1 = c + 1 < nchunks, more2 = c + 2 < nchunks;
        if (more1) {
          tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>((c + 1) * CHUNK), rb);
          prefetch_residual<kEpi, kTmaStore>(p, row, n0 + (c + 1) * CHUNK, resb);
        }
        process(ra, resa, c);
        if (more1) {
          tmem_ld_wait(rb);
          if (more2) {
            tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>((c + 2) * CHUNK), ra);
            prefetch_residual<kEpi, kTmaStore>(p, row, n0 + (c + 2) * CHUNK, resa);
          }
          process(rb, resb, c + 1);
          if (more2) tmem_ld_wait(ra);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&h.acc_empty[acc]);
      if (++acc == NUM_ACC) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (kTmaStore && lane == 0) bulk_wait_read<0>();
    if (p.out_amax != nullptr) {
      const uint32_t hb = __half_as_ushort(__float2half_rn(amax));
      const uint32_t bits = warp_max_u32(kSignedMax ? f16_order_key(hb) : hb);
      if (lane == 0 && bits != 0u) atomicMax(p.out_amax, bits);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, SK::TMEM_COLS);
  }
}


// ------------------------------------------------ resident amax + quantise
//
// Per-tensor quantise of a large fp16 tensor in ONE cooperative launch (one CTA
// per SM, all resident). Each CTA takes a contiguous slice, whose end stays on
// chip between the two phases: the last kResSmemVecs x 1024 16-byte vectors in
// shared memory (224 KB per SM, one bulk TMA copy) and the kResTmemVecs x 1024
// before them in tensor memory (all 512 columns of the SM's TMEM, 256 KB, with
// tcgen05.st / tcgen05.ld), 480 KB per SM, 71 MB over 148 SMs. Phase 1 reads
// the slice once for its amax: the bulk copy, then the TMEM part, then the rest
// of the slice (the front), last, so that it is the most recent data in L2.
// After one bounded grid-wide arrival agrees on the amax, phase 2 quantises
// the TMEM part, then re-reads the front from its end (the most recently read
// lines first), interleaved with the shared-memory part. The two kernels of
// the plain path (amax, then quantise) read the whole tensor from HBM twice.
// Codes, scale and amax bits are those of wbk_quantise_f16 (same scale rule,
// same element rule, same NaN handling).
constexpr int kResThreads = 1024;
constexpr int kResSmemVecs = 14;
constexpr int kResTmemVecs = 16;  // per thread: 64 TMEM columns of one lane
constexpr int kResUnroll = 4;     // 16-byte loads in flight per thread per step
constexpr size_t kResSmemBytes = static_cast<size_t>(kResSmemVecs) * kResThreads * 16;  // 224 KB
constexpr int64_t kResMinElems = int64_t{1} << 22;  // below this the plain two-pass quantiser is as fast
// Above this most of each slice's front misses L2 in phase 2 and the grid-wide
// arrival costs more than it saves (measured against the two-kernel pair on one
// box: 83.9M elements 69.8 against 73.7 us, 104.9M 92.8 against 89.3 us).
constexpr int64_t kResMaxElems = int64_t{88} << 20;
// Front vectors per CTA read with the evict_last hint: the last ~80 MB of the
// fronts (what L2 can keep for phase 2); earlier ones are read evict_first.
constexpr int64_t kResKeepVecs = 33792;

__device__ __forceinline__ void bulk_load_hint(void* smem, const void* gmem, uint32_t bytes, uint64_t* bar,
                                               uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(smem)),
      "l"(gmem), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

__device__ __forceinline__ void st_hint8(void* p, uint2 v, uint64_t pol) {
  asm volatile("st.global.L2::cache_hint.v2.u32 [%0], {%1, %2}, %3;" ::"l"(p), "r"(v.x), "r"(v.y), "l"(pol)
               : "memory");
}

// Two 16-byte vectors <-> 8 consecutive TMEM columns of this thread's lane
// (32x32b shape: thread i of the warp owns lane base+i). Warp-collective.
__device__ __forceinline__ void tmem_st_2v(uint32_t taddr, const uint4& a, const uint4& b) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w)
               : "memory");
}
__device__ __forceinline__ void tmem_ld_2v(uint32_t taddr, uint4& a, uint4& b) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(a.x), "=r"(a.y), "=r"(a.z), "=r"(a.w), "=r"(b.x), "=r"(b.y), "=r"(b.z), "=r"(b.w)
               : "r"(taddr)
               : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// Wait for this thread's tcgen05.ld; the loaded registers are tied to the wait
// so that no use of them moves above it.
__device__ __forceinline__ void tmem_ld_wait_8v(uint4 (&v)[8]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(v[0].x), "+r"(v[0].y), "+r"(v[0].z), "+r"(v[0].w), "+r"(v[1].x), "+r"(v[1].y), "+r"(v[1].z),
                 "+r"(v[1].w), "+r"(v[2].x), "+r"(v[2].y), "+r"(v[2].z), "+r"(v[2].w), "+r"(v[3].x), "+r"(v[3].y),
                 "+r"(v[3].z), "+r"(v[3].w), "+r"(v[4].x), "+r"(v[4].y), "+r"(v[4].z), "+r"(v[4].w), "+r"(v[5].x),
                 "+r"(v[5].y), "+r"(v[5].z), "+r"(v[5].w), "+r"(v[6].x), "+r"(v[6].y), "+r"(v[6].z), "+r"(v[6].w),
                 "+r"(v[7].x), "+r"(v[7].y), "+r"(v[7].z), "+r"(v[7].w)
               :
               : "memory");
}

// Phase 2 of quantise_resident_kernel. The TMEM part [t0, r0) first (warp-
// uniform: every thread runs the same tcgen05 instructions), then the front
// [v0, t0) from its end down, kResUnroll vectors per thread per step, with up
// to two of the shared-memory vectors ([r0, v1)) quantised between each step's
// loads and its stores; what is left of the shared-memory part at the end.
template <int kFmt, bool kFin>
__device__ __forceinline__ void resident_phase2(const uint4* __restrict__ x, uint2* __restrict__ q,
                                                const uint4* res_smem, uint32_t tmem_thr, int64_t v0, int64_t t0,
                                                int64_t r0, int64_t v1, float inv, float mx, uint64_t drop) {
  const int tid = threadIdx.x;
#pragma unroll
  for (int b = 0; b < kResTmemVecs / 8; ++b) {
    uint4 v[8];
    __syncwarp();  // converged (after the predicated stores of the batch before) for the warp-collective loads
#pragma unroll
    for (int u = 0; u < 4; ++u) tmem_ld_2v(tmem_thr + (b * 8 + 2 * u) * 4, v[2 * u], v[2 * u + 1]);
    tmem_ld_wait_8v(v);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int64_t i = t0 + static_cast<int64_t>(b * 8 + u) * kResThreads + tid;
      if (i < r0) st_hint8(q + i, q8x8<kFmt, kFin>(v[u], inv, mx), drop);
    }
  }
  int k = 0;  // next shared-memory vector of this thread
  auto smem_one = [&]() {
    const int64_t i = r0 + static_cast<int64_t>(k) * kResThreads + tid;
    if (i < v1) st_hint8(q + i, q8x8<kFmt, kFin>(res_smem[k * kResThreads + tid], inv, mx), drop);
    ++k;
  };
  int64_t j = t0 - 1 - tid;
  for (; j - (kResUnroll - 1) * kResThreads >= v0; j -= kResUnroll * kResThreads) {
    uint4 v[kResUnroll];
#pragma unroll
    for (int u = 0; u < kResUnroll; ++u) v[u] = ld_stream16_hint(x + j - u * kResThreads, drop);
    if (k < kResSmemVecs) smem_one();
    if (k < kResSmemVecs) smem_one();
#pragma unroll
    for (int u = 0; u < kResUnroll; ++u) st_hint8(q + j - u * kResThreads, q8x8<kFmt, kFin>(v[u], inv, mx), drop);
  }
  for (; j >= v0; j -= kResThreads) st_hint8(q + j, q8x8<kFmt, kFin>(ld_stream16_hint(x + j, drop), inv, mx), drop);
  while (k < kResSmemVecs) smem_one();
}

template <int kFmt>
__global__ void __launch_bounds__(kResThreads, 1)
quantise_resident_kernel(const uint4* __restrict__ x, int64_t nvec, float mx, uint2* __restrict__ q,
                         float* __restrict__ scale_out, uint32_t* __restrict__ amax_out, uint32_t* __restrict__ sync,
                         uint64_t timeout_ns) {
  extern __shared__ __align__(128) uint4 res_smem[];  // [kResSmemVecs][kResThreads], in slice order
  __shared__ uint32_t red[kResThreads / 32];
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t tmem_base_s;
  __shared__ uint32_t amax_s;
  __shared__ int ok_s;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t v0 = nvec * blockIdx.x / gridDim.x;
  const int64_t v1 = nvec * (blockIdx.x + 1) / gridDim.x;
  const int64_t r0 = v1 - min(v1 - v0, static_cast<int64_t>(kResSmemVecs) * kResThreads);  // shared memory [r0, v1)
  const int64_t t0 = r0 - min(r0 - v0, static_cast<int64_t>(kResTmemVecs) * kResThreads);  // TMEM [t0, r0)
  const uint32_t smem_bytes = static_cast<uint32_t>((v1 - r0) * 16);
  const uint64_t keep = l2_policy_evict_last(), drop = l2_policy_evict_first();
  // Under programmatic dependent launch: x may still be being written by the
  // grid before, and q read by it; a dependent grid may launch now (its CTAs
  // wait in griddepcontrol.wait until this grid has finished).
  griddep_wait();
  griddep_launch_dependents();
  if (tid == 0) {
    mbar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    if (smem_bytes != 0u) {
      mbar_arrive_expect_tx(&bar, smem_bytes);
      bulk_load_hint(res_smem, x + r0, smem_bytes, &bar, drop);
    } else {
      mbar_arrive(&bar);
    }
  }
  if (warp == 0) {  // all 512 columns: this CTA is alone on its SM (224 KB of shared memory)
    tmem_alloc(&tmem_base_s, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // This thread's 64 columns of its warp's lane quarter.
  const uint32_t tmem_thr = tmem_base_s + (static_cast<uint32_t>((warp & 3) * 32) << 16) +
                            static_cast<uint32_t>((warp >> 2) * (kResTmemVecs * 4));
  // Phase 1: the TMEM part (loaded, max-accumulated, stored to TMEM), then the front.
  uint32_t m2 = 0;  // packed running max of |x|
#pragma unroll
  for (int b = 0; b < kResTmemVecs / 8; ++b) {
    uint4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int64_t i = t0 + static_cast<int64_t>(b * 8 + u) * kResThreads + tid;
      v[u] = i < r0 ? ld_stream16_hint(x + i, drop) : make_uint4(0u, 0u, 0u, 0u);  // zeros change no max
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) m2 = absmax8_acc(m2, v[u]);
#pragma unroll
    for (int u = 0; u < 4; ++u) tmem_st_2v(tmem_thr + (b * 8 + 2 * u) * 4, v[2 * u], v[2 * u + 1]);
  }
  {
    const int64_t keep_from = t0 - kResKeepVecs;  // front vectors at or after it are read evict_last
    int64_t i = v0 + tid;
    for (; i + (kResUnroll - 1) * kResThreads < t0; i += kResUnroll * kResThreads) {
      const uint64_t pol = i >= keep_from ? keep : drop;
      uint4 v[kResUnroll];
#pragma unroll
      for (int u = 0; u < kResUnroll; ++u) v[u] = ld_stream16_hint(x + i + u * kResThreads, pol);
#pragma unroll
      for (int u = 0; u < kResUnroll; ++u) m2 = absmax8_acc(m2, v[u]);
    }
    for (; i < t0; i += kResThreads) m2 = absmax8_acc(m2, ld_stream16_hint(x + i, keep));
  }
  tmem_wait_st();
  int no_abort = 0;
  if (!mbar_wait(&bar, 0, &no_abort, timeout_ns, SITE_QUANT_SYNC)) {
    // The copy is still in flight: give it a short while more before the CTA goes on (the error is recorded).
    mbar_wait(&bar, 0, &no_abort, 1000000ull, SITE_DRAIN);
  }
  for (int k = 0; k < kResSmemVecs; ++k) {
    const int64_t i = r0 + static_cast<int64_t>(k) * kResThreads + tid;
    if (i < v1) m2 = absmax8_acc(m2, res_smem[k * kResThreads + tid]);
  }
  uint32_t m = warp_max_u32(absmax_lanes(m2));
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (tid == 0) {
    uint32_t mm = 0;
    for (int w = 0; w < kResThreads / 32; ++w) mm = max(mm, red[w]);
    if (mm != 0u) atomicMax(sync + 1, mm);
    const bool ok = grid_arrive_wait(sync + 0, gridDim.x, timeout_ns);
    amax_s = ok ? ld_acquire_gpu(sync + 1) : 0u;
    ok_s = ok ? 1 : 0;
    if (ok) {
      float sc, inv;
      scale_from_amax(amax_s, mx, sc, inv);
      if (blockIdx.x == 0) {
        if (scale_out != nullptr) *scale_out = sc;
        if (amax_out != nullptr) *amax_out = amax_s;
      }
      // Every CTA has read the amax once the last one leaves: reset the words for the next call.
      if (atomicAdd(sync + 2, 1u) == gridDim.x - 1u) {
        sync[0] = 0u;
        sync[1] = 0u;
        sync[2] = 0u;
      }
    }
  }
  __syncthreads();
  if (ok_s) {  // else the arrival gave up (recorded in the device error word)
    float sc, inv;
    scale_from_amax(amax_s, mx, sc, inv);
    if (inv != 0.0f)
      resident_phase2<kFmt, true>(x, q, res_smem, tmem_thr, v0, t0, r0, v1, inv, mx, drop);
    else  // an infinite amax
      resident_phase2<kFmt, false>(x, q, res_smem, tmem_thr, v0, t0, r0, v1, inv, mx, drop);
  }
  // Every path ends here: free the TMEM once all of this CTA's tcgen05.ld have completed.
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem_base_s, 512);
}

__global__ void selftest_wait_kernel(uint64_t timeout_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(&bar, 0, &abort_flag, timeout_ns, SITE_SELFTEST);  // nothing ever arrives
  __syncthreads();
}

// ------------------------------------------------------------------- host


// 2-D tensor map, inner dim contiguous.
int make_tmap(CUtensorMap* map, CUtensorMapDataType dtype, size_t elem_bytes, const void* base, uint64_t inner,
              uint64_t outer, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz) {
  auto encode = get_encode_fn();
  if (encode == nullptr) return fail(WBK_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {inner * elem_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(WBK_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return WBK_OK;
}


// Programmatic dependent launch of the GEMM (default on; WBK_PDL=0 turns it off).
bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("WBK_PDL");
    return e == nullptr || std::atoi(e) != 0;
  }();
  return on;
}

// Programmatic dependent launch for the cooperative (in-kernel quantise)
// variant too (default on; WBK_PDL_COOP=0 turns it off). A dependent grid can
// only launch once every CTA of the grid before it has started (and signalled),
// so that grid is wholly resident; the dependent's CTAs that find room wait in
// griddepcontrol.wait until it has finished, and the rest launch as its CTAs
// exit, so all of them are resident before any passes the wait. Measured on
// B200: the decoder-step linears 0.5 - 0.8 us shorter each.
bool pdl_coop_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("WBK_PDL_COOP");
    return !(e && e[0] == '0');
  }();
  return on;
}

template <int kBN, int kEpi, bool kTma, bool kPair, bool kQuantA, bool kResTma = false>
int launch_gemm(const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& to, const CUtensorMap& ta3,
                const CUtensorMap& tw3, const CUtensorMap& tr, const QuantParams& qp, int grid, cudaStream_t stream) {
  const KernelParams<kQuantA>& p = qp;
  static std::mutex mu;
  static std::vector<char> configured;
  const int dev = current_device();
  if (dev < 0) return fail(WBK_ERR_CUDA, "no current CUDA device");
  constexpr size_t kSmem = smem_bytes<kBN, kPair>();
  auto kernel = fp8_gemm_kernel<kBN, kEpi, kTma, kPair, kQuantA, kResTma>;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (static_cast<int>(configured.size()) <= dev) configured.resize(dev + 1, 0);
    if (!configured[dev]) {
      if (int e = cuda_check(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  static_cast<int>(kSmem)),
                             "cudaFuncSetAttribute(max dynamic smem)"))
        return e;
      configured[dev] = 1;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[3];
  int nattr = 0;
  // the kernel waits (griddep_wait) before reading anything a predecessor writes
  if (kQuantA ? pdl_coop_enabled() : pdl_enabled()) {
    attr[nattr].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[nattr].val.programmaticStreamSerializationAllowed = 1;
    ++nattr;
  }
  if (kQuantA) {  // the CTAs wait for one another: all must be resident at once
    attr[nattr].id = cudaLaunchAttributeCooperative;
    attr[nattr].val.cooperative = 1;
    ++nattr;
  }
  ResMap<kResTma> rm;
  if constexpr (kResTma) rm.map = tr;
  if (!kPair) {
    cfg.attrs = attr;
    cfg.numAttrs = nattr;
    return cuda_check(cudaLaunchKernelEx(&cfg, kernel, ta, tw, to, ta3, tw3, p, rm), "fp8 gemm launch");
  }
  {
    // Persistent pairs: never launch more clusters than can be resident at once.
    static std::vector<int> max_clusters;
    std::lock_guard<std::mutex> lock(mu);
    if (static_cast<int>(max_clusters.size()) <= dev) max_clusters.resize(dev + 1, -1);
    if (max_clusters[dev] < 0) {
      cudaLaunchConfig_t q = {};
      q.gridDim = cfg.gridDim;
      q.blockDim = dim3(THREADS, 1, 1);
      q.dynamicSmemBytes = kSmem;
      cudaLaunchAttribute qa[1];
      qa[0].id = cudaLaunchAttributeClusterDimension;
      qa[0].val.clusterDim.x = 2;
      qa[0].val.clusterDim.y = 1;
      qa[0].val.clusterDim.z = 1;
      q.attrs = qa;
      q.numAttrs = 1;
      int n = 0;
      if (int e = cuda_check(cudaOccupancyMaxActiveClusters(&n, kernel, &q), "cudaOccupancyMaxActiveClusters"))
        return e;
      if (n < 1) return fail(WBK_ERR_UNSUPPORTED, "fp8 gemm: no CTA pair fits on this device");
      max_clusters[dev] = n;
    }
    if (grid > 2 * max_clusters[dev]) cfg.gridDim.x = static_cast<unsigned>(2 * max_clusters[dev]);
  }
  attr[nattr].id = cudaLaunchAttributeClusterDimension;
  attr[nattr].val.clusterDim.x = 2;
  attr[nattr].val.clusterDim.y = 1;
  attr[nattr].val.clusterDim.z = 1;
  ++nattr;
  cfg.attrs = attr;
  cfg.numAttrs = nattr;
  return cuda_check(cudaLaunchKernelEx(&cfg, kernel, ta, tw, to, ta3, tw3, p, rm), "fp8 gemm (CTA pair) launch");
}

struct Maps {
  CUtensorMap a, w, out, a3, w3;
  CUtensorMap wh;   // skinny kernel: the weight box of a half-width item
  CUtensorMap res;  // CTA-pair residual epilogues: the residual, boxed like `out`
  bool res_tma = false;  // launch the TMA-residual variant (res is valid)
};

// TMA-loaded residual boxes in the CTA-pair residual epilogues (default on;
// WBK_GEMM_RES_TMA=0 keeps per-thread residual loads).
bool res_tma_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("WBK_GEMM_RES_TMA");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Five-K-block weight stages in the skinny kernel where they divide K (default on;
// WBK_SKINNY_G=2 keeps two-block stages).
bool skinny_g5_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("WBK_SKINNY_G");
    return !(e && e[0] == '2');
  }();
  return on;
}

// Half-width items in the skinny kernel's last round (default on; WBK_GEMM_HALF_TILES=0 turns them off).
bool half_items_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("WBK_GEMM_HALF_TILES");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Skinny kernel for M <= 64, K <= 1536 (default on; WBK_GEMM_SKINNY=0 uses the general kernel).
bool skinny_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("WBK_GEMM_SKINNY");
    return !(e && e[0] == '0');
  }();
  return on;
}

template <int kBN, int kEpi, bool kTma, bool kQuantA, int kG>
int launch_skinny(const Maps& m, const SkinnyParams& p, int grid, cudaStream_t stream) {
  static std::mutex mu;
  static std::vector<char> configured;
  const int dev = current_device();
  if (dev < 0) return fail(WBK_ERR_CUDA, "no current CUDA device");
  auto kernel = fp8_skinny_kernel<kBN, kEpi, kTma, kQuantA, kG>;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (static_cast<int>(configured.size()) <= dev) configured.resize(dev + 1, 0);
    if (!configured[dev]) {
      if (int e = cuda_check(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448),
                             "cudaFuncSetAttribute(max dynamic smem, skinny)"))
        return e;
      configured[dev] = 1;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.dynamicSmemBytes = skinny_smem(p.a_region, p.stages, Skinny<kBN, kG>::B_STAGE);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int nattr = 0;
  if (kQuantA ? pdl_coop_enabled() : pdl_enabled()) {
    attr[nattr].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[nattr].val.programmaticStreamSerializationAllowed = 1;
    ++nattr;
  }
  if (kQuantA) {  // the CTAs wait for one another: all must be resident at once
    attr[nattr].id = cudaLaunchAttributeCooperative;
    attr[nattr].val.cooperative = 1;
    ++nattr;
  }
  cfg.attrs = attr;
  cfg.numAttrs = nattr;
  return cuda_check(cudaLaunchKernelEx(&cfg, kernel, m.a, m.w, m.out, m.a3, m.w3, m.wh, p), "fp8 skinny gemm launch");
}

template <int kBN, bool kQuantA, int kG>
int dispatch_skinny(int epilogue, bool tma, const Maps& m, const SkinnyParams& p, int grid, cudaStream_t s) {
#define WBK_SK(E) \
  return tma ? launch_skinny<kBN, E, true, kQuantA, kG>(m, p, grid, s) : launch_skinny<kBN, E, false, kQuantA, kG>(m, p, grid, s)
  switch (epilogue) {
    case WBK_EPI_NONE: WBK_SK(WBK_EPI_NONE);
    case WBK_EPI_GELU: WBK_SK(WBK_EPI_GELU);
    case WBK_EPI_RESIDUAL: WBK_SK(WBK_EPI_RESIDUAL);
    case WBK_EPI_RESIDUAL_CLAMP: WBK_SK(WBK_EPI_RESIDUAL_CLAMP);
    default: WBK_SK(WBK_EPI_BIAS_MAXKEY);
  }
#undef WBK_SK
}

template <int kBN, int kEpi, bool kPair, bool kQuantA>
int dispatch_store(bool tma, const Maps& m, const QuantParams& p, int grid, cudaStream_t s) {
  if constexpr (kPair && has_residual(kEpi)) {
    if (tma && m.res_tma)
      return launch_gemm<kBN, kEpi, true, kPair, kQuantA, true>(m.a, m.w, m.out, m.a3, m.w3, m.res, p, grid, s);
  }
  return tma ? launch_gemm<kBN, kEpi, true, kPair, kQuantA>(m.a, m.w, m.out, m.a3, m.w3, m.res, p, grid, s)
             : launch_gemm<kBN, kEpi, false, kPair, kQuantA>(m.a, m.w, m.out, m.a3, m.w3, m.res, p, grid, s);
}

template <int kBN, bool kPair = false, bool kQuantA = false>
int dispatch_epi(int epilogue, bool tma, const Maps& m, const QuantParams& p, int grid, cudaStream_t s) {
  switch (epilogue) {
    case WBK_EPI_NONE: return dispatch_store<kBN, WBK_EPI_NONE, kPair, kQuantA>(tma, m, p, grid, s);
    case WBK_EPI_GELU: return dispatch_store<kBN, WBK_EPI_GELU, kPair, kQuantA>(tma, m, p, grid, s);
    case WBK_EPI_RESIDUAL: return dispatch_store<kBN, WBK_EPI_RESIDUAL, kPair, kQuantA>(tma, m, p, grid, s);
    case WBK_EPI_RESIDUAL_CLAMP:
      return dispatch_store<kBN, WBK_EPI_RESIDUAL_CLAMP, kPair, kQuantA>(tma, m, p, grid, s);
    default: return dispatch_store<kBN, WBK_EPI_BIAS_MAXKEY, kPair, kQuantA>(tma, m, p, grid, s);
  }
}

// 3-D view of a row-major [rows, K] fp8 matrix as (128 bytes of K, rows, K / 128 blocks)
// with a box of (128, box_rows, g): one load brings g consecutive K blocks, each a
// [box_rows x 128 B] 128-byte-swizzled block, stacked in shared memory. Needs K % 128 == 0
// (a partial last block would read past the row end instead of zero-filling).
int make_tmap_kblocks(CUtensorMap* map, const void* base, uint64_t K, uint64_t rows, uint32_t box_rows, uint32_t g) {
  auto encode = get_encode_fn();
  if (encode == nullptr) return fail(WBK_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(BK), rows, K / BK};
  const cuuint64_t strides[2] = {K, static_cast<cuuint64_t>(BK)};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(BK), box_rows, g};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(WBK_ERR_CUDA, "cuTensorMapEncodeTiled (K blocks) failed (%d)", static_cast<int>(r));
  return WBK_OK;
}

// One 3-D TMA load per operand per stage (default on; WBK_GEMM_GROUPED=0 issues
// the stage's K blocks as separate 2-D loads).
bool kblocks_grouping_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("WBK_GEMM_GROUPED");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Narrow items for a CTA-pair GEMM's partial last round (default on; WBK_GEMM_NARROW=0 keeps whole tiles).
bool narrow_tail_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("WBK_GEMM_NARROW");
    return !(e && e[0] == '0');
  }();
  return on;
}

bool pair_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("WBK_GEMM_PAIR");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Tile width. Short-M GEMMs (the decoder step) are weight-streaming and
// HBM-bound: 64-wide tiles spread the weight over every SM. Otherwise the
// choice is 256-wide tiles on CTA pairs or 128-wide tiles on single CTAs, by
// rounds of tiles: measured on B200, a CTA computing a 128 x 128 tile does
// ~0.63 of the work of a pair round (256 x 256 on two SMs) in the same time
// per SM — the pair halves each SM's operand traffic per FLOP, which is what
// limits it — so pairs win unless they leave too many SMs idle in their last
// round (1500 x 5120 x 1280: 2 pair rounds beat 4 single-CTA rounds by 11 %).
int pick_bn(int64_t M, int64_t N, int sms) {
  static const int forced = [] {  // WBK_GEMM_BN=64|128|256 overrides the choice (tuning)
    const char* e = std::getenv("WBK_GEMM_BN");
    const int v = e ? std::atoi(e) : 0;
    return (v == 64 || v == 128 || v == 256) ? v : 0;
  }();
  if (forced) return forced;
  if (M <= BM) return 64;
  const int64_t pairs = sms / 2 > 0 ? sms / 2 : 1;
  const int64_t pair_tiles = ((M + 2 * BM - 1) / (2 * BM)) * ((N + 255) / 256);
  const int64_t single_tiles = ((M + BM - 1) / BM) * ((N + 127) / 128);
  const int64_t pair_rounds = (pair_tiles + pairs - 1) / pairs;
  const int64_t single_rounds = (single_tiles + sms - 1) / sms;
  return 100 * pair_rounds <= 65 * single_rounds ? 256 : 128;
}

// The ticket block has one fixed size for every shape (split-K needs 2 * tiles <= SMs,
// so at most 512 tiles), so the partials of one shape never overlap the tickets of
// another sharing the workspace.
constexpr int kMaxSplitTiles = 512;
// Split-K plan for short-M GEMMs (64-wide tiles): K slices per tile so the
// (tile, slice) work items cover the SMs. Measured on B200, splitting pays only
// when each CTA would otherwise stream a long K for very few rows (M <= 32,
// K >= 2048, at least 4 K blocks per slice: M = 16 or 1, N = 1280, K = 5120 ran
// ~7 % faster); at M = 64 the fp32 partial round trip costs more than the
// shorter K loop saves (N = 1280, K = 5120: 24.6 us split vs 17.7 us), so the
// plan is 1 there.
// WBK_SPLITK = auto (default: the measured rule above) | off | max (split whenever
// the tiles leave half the SMs idle, one stage per slice at least; for tuning).
int splitk_mode() {
  static const int mode = [] {
    const char* e = std::getenv("WBK_SPLITK");
    if (e == nullptr) return 0;
    const std::string v(e);
    return v == "off" ? 1 : (v == "max" ? 2 : 0);
  }();
  return mode;
}

void splitk_plan(int64_t M, int64_t N, int64_t K, int* splits, int* tiles) {
  *splits = 1;
  *tiles = 0;
  const int mode = splitk_mode();
  if (M <= 0 || N <= 0 || K <= 0 || M > (mode == 2 ? BM : 32) || mode == 1) return;
  const int sms = sm_count() > 0 ? sm_count() : 148;
  const int64_t t = (N + 63) / 64;
  const int64_t kblocks = (K + BK - 1) / BK;
  const int64_t stages = (kblocks + Tile<64>::G - 1) / Tile<64>::G;
  *tiles = static_cast<int>(t);
  if (2 * t > sms || t > kMaxSplitTiles || (mode == 0 && kblocks < 16)) return;
  int64_t sp = sms / t;
  if (sp > stages) sp = stages;
  if (sp > 16) sp = 16;
  *splits = static_cast<int>(sp < 1 ? 1 : sp);
}
int64_t splitk_ticket_bytes(int /*tiles*/) { return static_cast<int64_t>(kMaxSplitTiles) * EPI_WARPS * 4; }
// Workspace layout: [kSyncBytes: the in-kernel quantise's sync words][split-K
// tickets][split-K partials]; every word is back at zero when a call ends.
constexpr int64_t kSyncBytes = 256;
int64_t splitk_ws_bytes(int splits, int tiles) {
  if (splits <= 1) return 0;
  return kSyncBytes + splitk_ticket_bytes(tiles) + static_cast<int64_t>(tiles) * splits * BM * 64 * 4;
}

// In-kernel activation quantise of wbk_linear_fp8_f16 (default on;
// WBK_LINEAR_FUSED=0 runs the quantiser kernel and then the GEMM instead).
bool linear_fused_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("WBK_LINEAR_FUSED");
    return !(e && e[0] == '0');
  }();
  return on;
}

// The fp16 activation side of wbk_linear_fp8_f16 when the GEMM quantises A itself.
struct QuantIn {
  const void* a16;
  int a_fmt;
  void* a_q;
  float* scale_out;
  uint32_t* amax_out;
};

int gemm_impl(const void* A, const void* W, int64_t M, int64_t N, int64_t K, int a_fmt, int w_fmt, float alpha,
              const float* a_scale, const float* w_scale, const void* bias, const void* residual, void* out,
              int epilogue, uint32_t* out_amax_bits, void* workspace, int64_t workspace_bytes, cudaStream_t s,
              const QuantIn* qin);

}  // namespace
}  // namespace wbk

using namespace wbk;

extern "C" {

int64_t wbk_gemm_fp8_ws_bytes(int64_t M, int64_t N, int64_t K) {
  if (M <= 0) return 0;
  int splits = 0, tiles = 0;
  splitk_plan(M, N, K, &splits, &tiles);
  int64_t need = splitk_ws_bytes(splits, tiles);
  if (M <= BM && need < kSyncBytes) need = kSyncBytes;  // wbk_linear_fp8_f16's quantise sync words
  return need;
}

int wbk_gemm_fp8(const void* A, const void* W, int64_t M, int64_t N, int64_t K, int a_fmt, int w_fmt, float alpha,
                 const float* a_scale, const float* w_scale, const void* bias, const void* residual, void* out,
                 int epilogue, uint32_t* out_amax_bits, wbk_stream_t stream) {
  return wbk_gemm_fp8_ws(A, W, M, N, K, a_fmt, w_fmt, alpha, a_scale, w_scale, bias, residual, out, epilogue,
                         out_amax_bits, nullptr, 0, stream);
}

int wbk_gemm_fp8_ws(const void* A, const void* W, int64_t M, int64_t N, int64_t K, int a_fmt, int w_fmt, float alpha,
                    const float* a_scale, const float* w_scale, const void* bias, const void* residual, void* out,
                    int epilogue, uint32_t* out_amax_bits, void* workspace, int64_t workspace_bytes,
                    wbk_stream_t stream) {
  return gemm_impl(A, W, M, N, K, a_fmt, w_fmt, alpha, a_scale, w_scale, bias, residual, out, epilogue, out_amax_bits,
                   workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream), nullptr);
}

int wbk_linear_fp8_f16(const void* A16, int64_t M, int64_t N, int64_t K, int a_fmt, void* a_q_out, float* a_scale_out,
                       uint32_t* a_amax_ws, const void* W, int w_fmt, const float* w_scale, float alpha,
                       const void* bias, const void* residual, void* out, int epilogue, uint32_t* out_amax_bits,
                       void* workspace, int64_t workspace_bytes, wbk_stream_t stream) {
  if (a_fmt != WBK_FMT_E4M3 && a_fmt != WBK_FMT_E5M2)
    return fail(WBK_ERR_INVALID_ARG, "wbk_linear_fp8_f16: unknown fp8 format %d", a_fmt);
  if (a_scale_out == nullptr || a_amax_ws == nullptr)
    return fail(WBK_ERR_INVALID_ARG, "wbk_linear_fp8_f16: a_scale_out and a_amax_ws are required");
  if (M < 0 || N <= 0 || K <= 0 || M > INT32_MAX || K > INT32_MAX)
    return fail(WBK_ERR_INVALID_ARG, "wbk_linear_fp8_f16: bad shape M=%lld N=%lld K=%lld", (long long)M, (long long)N,
                (long long)K);
  if (M > 0 && (A16 == nullptr || a_q_out == nullptr))
    return fail(WBK_ERR_INVALID_ARG, "wbk_linear_fp8_f16: null activation pointer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool fused = linear_fused_enabled() && M > 0 && M <= BM && K % 16 == 0 && aligned(A16, 16) &&
                     aligned(a_q_out, 16) && workspace != nullptr;
  if (fused) {
    const QuantIn q{A16, a_fmt, a_q_out, a_scale_out, a_amax_ws};
    return gemm_impl(a_q_out, W, M, N, K, a_fmt, w_fmt, alpha, nullptr, w_scale, bias, residual, out, epilogue,
                     out_amax_bits, workspace, workspace_bytes, s, &q);
  }
  // Two launches: the quantiser kernel, then the GEMM on its codes and scale.
  if (int e = wbk_quantise_f16(A16, M * K, a_fmt, a_q_out, a_scale_out, a_amax_ws, stream)) return e;
  return gemm_impl(a_q_out, W, M, N, K, a_fmt, w_fmt, alpha, a_scale_out, w_scale, bias, residual, out, epilogue,
                   out_amax_bits, workspace, workspace_bytes, s, nullptr);
}

}  // extern "C"

namespace wbk {
namespace {

int gemm_impl(const void* A, const void* W, int64_t M, int64_t N, int64_t K, int a_fmt, int w_fmt, float alpha,
              const float* a_scale, const float* w_scale, const void* bias, const void* residual, void* out,
              int epilogue, uint32_t* out_amax_bits, void* workspace, int64_t workspace_bytes, cudaStream_t s,
              const QuantIn* qin) {
  if (M < 0 || N <= 0 || K <= 0)
    return fail(WBK_ERR_INVALID_ARG, "wbk_gemm_fp8: bad shape M=%lld N=%lld K=%lld", (long long)M, (long long)N,
                (long long)K);
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX || M * N > (int64_t(1) << 46))
    return fail(WBK_ERR_UNSUPPORTED, "wbk_gemm_fp8: shape too large");
  if (K % 16 != 0) return fail(WBK_ERR_UNSUPPORTED, "wbk_gemm_fp8: K=%lld must be a multiple of 16 (TMA row pitch)", (long long)K);
  if ((a_fmt != WBK_FMT_E4M3 && a_fmt != WBK_FMT_E5M2) || (w_fmt != WBK_FMT_E4M3 && w_fmt != WBK_FMT_E5M2))
    return fail(WBK_ERR_INVALID_ARG, "wbk_gemm_fp8: unknown fp8 format");
  if (epilogue < WBK_EPI_NONE || epilogue > WBK_EPI_BIAS_MAXKEY)
    return fail(WBK_ERR_INVALID_ARG, "wbk_gemm_fp8: unknown epilogue %d", epilogue);
  const bool needs_res = epilogue == WBK_EPI_RESIDUAL || epilogue == WBK_EPI_RESIDUAL_CLAMP;
  if (needs_res && residual == nullptr) return fail(WBK_ERR_INVALID_ARG, "wbk_gemm_fp8: residual epilogue without residual");
  if (epilogue == WBK_EPI_BIAS_MAXKEY && out_amax_bits == nullptr)
    return fail(WBK_ERR_INVALID_ARG, "wbk_gemm_fp8: the max-key epilogue needs out_amax_bits");
  if (M == 0) return WBK_OK;
  if (A == nullptr || W == nullptr || out == nullptr) return fail(WBK_ERR_INVALID_ARG, "wbk_gemm_fp8: null pointer");
  if (!aligned(A, 16) || !aligned(W, 16)) return fail(WBK_ERR_UNSUPPORTED, "wbk_gemm_fp8: A and W must be 16-byte aligned");
  if (!aligned(out, 2) || (bias && !aligned(bias, 2)) || (residual && !aligned(residual, 2)))
    return fail(WBK_ERR_INVALID_ARG, "wbk_gemm_fp8: fp16 pointers must be 2-byte aligned");

  // TMA store and vector loads need 16-byte aligned rows: N % 8 == 0 and aligned bases.
  const bool vec = (N % 8 == 0) && aligned(out, 16) && (!bias || aligned(bias, 16)) && (!residual || aligned(residual, 16));

  Maps maps;
  CUtensorMap& ta = maps.a;
  CUtensorMap& tw = maps.w;
  CUtensorMap& to = maps.out;
  // M <= 64 (decoder step): load a 64-row A box; the MMA still reads 128 rows, and
  // TMEM lanes 64..127 (computed from stale shared memory) are never stored.
  const uint32_t a_box_rows = M <= 64 ? 64u : static_cast<uint32_t>(BM);
  if (int e = make_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, A, K, M, BK, a_box_rows, CU_TENSOR_MAP_SWIZZLE_128B))
    return e;
  const int sms = sm_count() > 0 ? sm_count() : 148;
  const int bn = pick_bn(M, N, sms);
  // Large GEMMs run on CTA pairs (256 x 256 tiles, each CTA loading half of the weight rows).
  const bool pair = bn == 256 && pair_enabled() && sms >= 2;
  const uint32_t w_box_rows = static_cast<uint32_t>(pair ? bn / 2 : bn);
  if (int e = make_tmap(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, W, K, N, BK, w_box_rows, CU_TENSOR_MAP_SWIZZLE_128B))
    return e;
  if (vec) {
    if (int e = make_tmap(&to, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, out, N, M, CHUNK, 32, CU_TENSOR_MAP_SWIZZLE_64B))
      return e;
  } else {
    to = ta;  // unused by the direct-store kernel
  }
  // Skinny path (A resident, weight-only ring): M <= 64, K <= 1536, no K split;
  // used where it measured faster on B200: the in-kernel quantise (its early
  // weight ring is deeper) and shapes with more tiles than SMs (A is not
  // re-read per tile: 64 x 51866 x 1280 in 24.2 us against 26.4). With one
  // tile per CTA its smaller weight stages cost ~0.4 us more than the general
  // kernel's.
  const int64_t kblocks_all = (K + BK - 1) / BK;
  const int64_t tiles_if_skinny = (N + bn - 1) / bn;
  bool skinny = skinny_enabled() && M <= kSkRows && !pair && (bn == 64 || bn == 128) &&
                kblocks_all <= kSkMaxKBlocks && (qin != nullptr || tiles_if_skinny > sms);
  if (skinny && workspace != nullptr) {
    int sp = 1, st = 0;
    splitk_plan(M, N, K, &sp, &st);
    skinny = sp == 1;
  }
  const uint32_t sk_region = static_cast<uint32_t>(kblocks_all * kSkABlock + kSkASlack);
  // 5 K blocks per weight stage when they divide K (64-wide tiles), else 2.
  const bool sk_g5 = bn == 64 && kblocks_all % 5 == 0 && skinny_g5_enabled();
  const int sk_g = sk_g5 ? 5 : 2;
  const int sk_bstage = bn == 64 ? (sk_g5 ? Skinny<64, 5>::B_STAGE : Skinny<64>::B_STAGE) : Skinny<128>::B_STAGE;
  int sk_stages = 0;
  if (skinny) {
    const int64_t avail = 232448 - static_cast<int64_t>(skinny_smem(sk_region, 0, sk_bstage));
    sk_stages = static_cast<int>(avail / sk_bstage);
    if (sk_stages > kSkMaxStages) sk_stages = kSkMaxStages;
    skinny = sk_stages >= 2;
  }
  // One 3-D load per operand per stage when K is a whole number of 128-byte blocks
  // (the skinny kernel: two K blocks per box for A and for each W stage).
  const int group = bn == 64 ? Tile<64>::G : (pair ? Tile<256, true>::G : Tile<128>::G);
  const int a_group = skinny ? 2 : group;  // the skinny kernel loads A two K blocks per box
  const int w_group = skinny ? sk_g : group;
  bool grouped = K % BK == 0 && kblocks_grouping_enabled();
  if (grouped) {
    // If the driver does not take the blocked view, fall back to per-block 2-D loads.
    grouped = make_tmap_kblocks(&maps.a3, A, static_cast<uint64_t>(K), static_cast<uint64_t>(M), a_box_rows,
                                static_cast<uint32_t>(a_group)) == WBK_OK &&
              make_tmap_kblocks(&maps.w3, W, static_cast<uint64_t>(K), static_cast<uint64_t>(N), w_box_rows,
                                static_cast<uint32_t>(w_group)) == WBK_OK;
  }
  if (!grouped) {
    maps.a3 = ta;  // unused: the kernel issues per-block 2-D loads
    maps.w3 = tw;
  }

  QuantParams p{};  // zeroed: fields a path does not use stay 0
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  const int tile_rows = pair ? 2 * BM : BM;
  const int tiles_m = static_cast<int>((M + tile_rows - 1) / tile_rows);
  p.tiles_n = static_cast<int>((N + bn - 1) / bn);
  const int64_t num_tiles = static_cast<int64_t>(tiles_m) * p.tiles_n;
  if (num_tiles > INT32_MAX) return fail(WBK_ERR_UNSUPPORTED, "wbk_gemm_fp8: too many tiles");
  p.num_tiles = static_cast<int>(num_tiles);
  p.kblocks = static_cast<int>((K + BK - 1) / BK);
  // Split-K for the narrow-tile (short-M) shapes when the caller gave a workspace.
  p.splits = 1;
  p.ws_partials = nullptr;
  p.ws_tickets = nullptr;
  if (workspace != nullptr && !aligned(workspace, 256))
    return fail(WBK_ERR_INVALID_ARG, "wbk_gemm_fp8_ws: workspace must be 256-byte aligned");
  if (qin != nullptr && workspace_bytes < kSyncBytes)
    return fail(WBK_ERR_INVALID_ARG, "wbk_linear_fp8_f16: workspace of %lld bytes, needs %lld",
                (long long)workspace_bytes, (long long)kSyncBytes);
  if (workspace != nullptr && !pair && bn == 64) {
    int splits = 1, tiles = 0;
    splitk_plan(M, N, K, &splits, &tiles);
    const int64_t need = splitk_ws_bytes(splits, tiles);
    if (splits > 1) {
      if (workspace_bytes < need)
        return fail(WBK_ERR_INVALID_ARG, "wbk_gemm_fp8_ws: workspace of %lld bytes, needs %lld",
                    (long long)workspace_bytes, (long long)need);
      p.splits = splits;
      p.ws_tickets = reinterpret_cast<uint32_t*>(static_cast<char*>(workspace) + kSyncBytes);
      p.ws_partials =
          reinterpret_cast<float*>(static_cast<char*>(workspace) + kSyncBytes + splitk_ticket_bytes(tiles));
    }
  }
  p.a_f16 = nullptr;
  p.a_q = nullptr;
  p.a_scale_out = nullptr;
  p.a_amax_out = nullptr;
  p.qsync = nullptr;
  p.a_vecs = 0;
  p.a_max_fp8 = 0.0f;
  p.a_e5m2 = 0;
  if (qin != nullptr) {
    if (!skinny && (bn != 64 || pair))
      return fail(WBK_ERR_UNSUPPORTED, "wbk_linear_fp8_f16: in-kernel quantise needs M <= 128");
    p.a_f16 = static_cast<const __half*>(qin->a16);
    p.a_q = static_cast<uint8_t*>(qin->a_q);
    p.a_scale_out = qin->scale_out;
    p.a_amax_out = qin->amax_out;
    p.qsync = static_cast<uint32_t*>(workspace);
    p.a_vecs = M * K / 8;
    p.a_max_fp8 = fmt_max(qin->a_fmt);
    p.a_e5m2 = qin->a_fmt == WBK_FMT_E5M2 ? 1 : 0;
  }
  p.num_items = p.num_tiles * p.splits;
  p.full_items = p.num_items;  // CTA pairs may narrow their last round below
  p.narrow_shift = 0;
  p.alpha = alpha;
  p.a_scale = a_scale;
  p.w_scale = w_scale;
  p.bias = static_cast<const __half*>(bias);
  p.residual = static_cast<const __half*>(residual);
  p.out = static_cast<__half*>(out);
  p.out_amax = out_amax_bits;
  p.out_pairs = (N % 2 == 0) && aligned(out, 4);
  p.a_box_bytes = a_box_rows * BK;
  p.grouped = grouped ? 1 : 0;
  // Instruction descriptor (kind::f8f6f4): D fp32 [4,6)=1; A format [7,10);
  // B format [10,13); both K-major (bits 15,16 = 0); N>>3 [17,23); M>>4 [24,29).
  p.idesc = (1u << 4) | (static_cast<uint32_t>(a_fmt) << 7) | (static_cast<uint32_t>(w_fmt) << 10) |
            (static_cast<uint32_t>(bn >> 3) << 17) | (static_cast<uint32_t>(tile_rows >> 4) << 24);
  p.timeout_ns = wait_timeout_ns();

  if (pair) {
    // Residual epilogues with TMA stores also load the residual by TMA (same box and swizzle).
    if (needs_res && vec && res_tma_enabled()) {
      if (int e = make_tmap(&maps.res, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, residual, N, M, CHUNK, 32,
                            CU_TENSOR_MAP_SWIZZLE_64B))
        return e;
      maps.res_tma = true;
    } else {
      maps.res = to;  // unused
    }
    const int pairs = sms / 2;
    // Last round: when the tiles past the whole rounds would leave most pairs idle, split
    // each of them into 2 or 4 narrower items (all in one round). A narrow item costs more
    // than its share of a tile (its A rows are loaded whole), but the round ends sooner.
    if (narrow_tail_enabled()) {
      const int64_t full = (num_tiles / pairs) * pairs;
      const int64_t left = num_tiles - full;
      const int shift = left == 0 ? 0 : (4 * left <= pairs ? 2 : (2 * left <= pairs ? 1 : 0));
      if (shift > 0) {
        // weight boxes of a narrow item: (128 >> shift) rows per CTA, in the slot the kernel
        // does not otherwise read (tmap_w with grouped loads, tmap_w3 without)
        const uint32_t rows_n = w_box_rows >> shift;
        const int e = grouped ? make_tmap_kblocks(&maps.w, W, static_cast<uint64_t>(K), static_cast<uint64_t>(N),
                                                  rows_n, static_cast<uint32_t>(group))
                              : make_tmap(&maps.w3, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, W, K, N, BK, rows_n,
                                          CU_TENSOR_MAP_SWIZZLE_128B);
        if (e != WBK_OK) return e;
        p.full_items = static_cast<int>(full);
        p.narrow_shift = shift;
        p.num_items = static_cast<int>(full + (left << shift));
      }
    }
    const int grid = 2 * (p.num_items < pairs ? p.num_items : pairs);
    return dispatch_epi<256, true>(epilogue, vec, maps, p, grid, s);
  }
  const int grid = p.num_items < sms ? p.num_items : sms;
  if (skinny) {
    SkinnyParams sp;
    static_cast<QuantParams&>(sp) = p;
    sp.stages = sk_stages;
    sp.a_region = sk_region;
    sp.a_grouped = grouped ? 1 : 0;
    // Half-width items for the last round when whole tiles would leave part of it
    // idle: e.g. 811 tiles on 148 CTAs (71 CTAs with a sixth tile) become 740
    // whole tiles and 141 half tiles, one each on 141 CTAs.
    sp.full_items = sp.num_tiles;
    sp.idesc_half = (p.idesc & ~(0x3Fu << 17)) | (static_cast<uint32_t>((bn / 2) >> 3) << 17);
    maps.wh = maps.w3;  // unused unless there are half items
    if (sp.num_tiles > grid && sp.num_tiles % grid != 0 && half_items_enabled()) {
      const int full = (sp.num_tiles / grid) * grid;
      const int64_t rest = N - static_cast<int64_t>(full) * bn;
      const int halves = static_cast<int>((rest + bn / 2 - 1) / (bn / 2));
      if (halves <= grid) {
        const uint32_t half_rows = static_cast<uint32_t>(bn / 2);
        const int e = grouped ? make_tmap_kblocks(&maps.wh, W, static_cast<uint64_t>(K), static_cast<uint64_t>(N),
                                                  half_rows, static_cast<uint32_t>(sk_g))
                              : make_tmap(&maps.wh, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, W, K, N, BK, half_rows,
                                          CU_TENSOR_MAP_SWIZZLE_128B);
        if (e != WBK_OK) return e;
        sp.full_items = full;
        sp.num_tiles = full + halves;
        sp.num_items = sp.num_tiles;
      }
    }
    if (bn == 64 && sk_g5) return qin ? dispatch_skinny<64, true, 5>(epilogue, vec, maps, sp, grid, s)
                                      : dispatch_skinny<64, false, 5>(epilogue, vec, maps, sp, grid, s);
    if (bn == 64) return qin ? dispatch_skinny<64, true, 2>(epilogue, vec, maps, sp, grid, s)
                             : dispatch_skinny<64, false, 2>(epilogue, vec, maps, sp, grid, s);
    return qin ? dispatch_skinny<128, true, 2>(epilogue, vec, maps, sp, grid, s)
               : dispatch_skinny<128, false, 2>(epilogue, vec, maps, sp, grid, s);
  }
  if (qin != nullptr) return dispatch_epi<64, false, true>(epilogue, vec, maps, p, grid, s);
  if (bn == 64) return dispatch_epi<64>(epilogue, vec, maps, p, grid, s);
  if (bn == 128) return dispatch_epi<128>(epilogue, vec, maps, p, grid, s);
  return dispatch_epi<256>(epilogue, vec, maps, p, grid, s);
}

}  // namespace
}  // namespace wbk

extern "C" {

int wbk_device_error(uint32_t* code_out) {
  if (code_out == nullptr) return fail(WBK_ERR_INVALID_ARG, "wbk_device_error: null pointer");
  if (int e = cuda_check(cudaDeviceSynchronize(), "wbk_device_error synchronize")) return e;
  uint32_t v = 0, va = 0;
  if (int e = cuda_check(cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v)), "wbk_device_error read")) return e;
  const uint32_t zero = 0;
  if (int e = cuda_check(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero)), "wbk_device_error clear")) return e;
  if (int e = attn_read_device_error(&va, true)) return e;
  *code_out = v != 0 ? v : va;  // the GEMM unit's word first, then the attention unit's
  return WBK_OK;
}

int wbk_quantise_f16_resident(const void* x, int64_t n, int fmt, void* q_out, float* scale_out, uint32_t* amax_ws,
                              uint32_t* sync_ws, wbk_stream_t stream) {
  using namespace wbk;
  if (fmt != WBK_FMT_E4M3 && fmt != WBK_FMT_E5M2)
    return fail(WBK_ERR_INVALID_ARG, "wbk_quantise_f16_resident: fmt must be WBK_FMT_E4M3 or WBK_FMT_E5M2");
  if (amax_ws == nullptr) return fail(WBK_ERR_INVALID_ARG, "wbk_quantise_f16_resident: amax_ws is null");
  if (n < 0) return fail(WBK_ERR_INVALID_ARG, "wbk_quantise_f16_resident: n < 0");
  if (n > 0 && (x == nullptr || q_out == nullptr))
    return fail(WBK_ERR_INVALID_ARG, "wbk_quantise_f16_resident: null pointer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool resident = sync_ws != nullptr && n >= kResMinElems && n <= kResMaxElems && n % 8 == 0 && aligned(x, 16) &&
                        aligned(q_out, 8) &&
                        aligned(sync_ws, 16);
  if (!resident) return wbk_quantise_f16(x, n, fmt, q_out, scale_out, amax_ws, stream);
  int dev = 0;
  if (int e = cuda_check(cudaGetDevice(&dev), "cudaGetDevice")) return e;
  {
    static std::mutex mu;
    static std::vector<char> configured;
    std::lock_guard<std::mutex> lock(mu);
    if (static_cast<int>(configured.size()) <= dev) configured.resize(dev + 1, 0);
    if (!configured[dev]) {
      for (const void* k : {reinterpret_cast<const void*>(&quantise_resident_kernel<WBK_FMT_E4M3>),
                            reinterpret_cast<const void*>(&quantise_resident_kernel<WBK_FMT_E5M2>)})
        if (int e = cuda_check(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                    static_cast<int>(kResSmemBytes)),
                               "cudaFuncSetAttribute(max dynamic smem, resident quantise)"))
          return e;
      configured[dev] = 1;
    }
  }
  const int sms = sm_count() > 0 ? sm_count() : 148;
  const int64_t nvec = n / 8;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(sms), 1, 1);
  cfg.blockDim = dim3(kResThreads, 1, 1);
  cfg.dynamicSmemBytes = kResSmemBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int nattr = 0;
  attr[nattr].id = cudaLaunchAttributeCooperative;  // the CTAs wait for one another: all must be resident at once
  attr[nattr].val.cooperative = 1;
  ++nattr;
  if (pdl_coop_enabled()) {  // the kernel waits (griddep_wait) before touching memory
    attr[nattr].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[nattr].val.programmaticStreamSerializationAllowed = 1;
    ++nattr;
  }
  cfg.attrs = attr;
  cfg.numAttrs = nattr;
  const uint4* xv = static_cast<const uint4*>(x);
  uint2* qv = static_cast<uint2*>(q_out);
  const float mx = fmt == WBK_FMT_E4M3 ? 448.0f : 57344.0f;
  const uint64_t timeout = wait_timeout_ns();
  cudaError_t err = fmt == WBK_FMT_E4M3
                        ? cudaLaunchKernelEx(&cfg, quantise_resident_kernel<WBK_FMT_E4M3>, xv, nvec, mx, qv, scale_out,
                                             amax_ws, sync_ws, timeout)
                        : cudaLaunchKernelEx(&cfg, quantise_resident_kernel<WBK_FMT_E5M2>, xv, nvec, mx, qv, scale_out,
                                             amax_ws, sync_ws, timeout);
  if (err == cudaErrorCooperativeLaunchTooLarge) {
    // Not every SM can hold one of its CTAs right now (the device is shared, or partitioned): the
    // two-kernel path gives the same codes, scale and amax.
    (void)cudaGetLastError();
    return wbk_quantise_f16(x, n, fmt, q_out, scale_out, amax_ws, stream);
  }
  return cuda_check(err, "wbk_quantise_f16_resident launch");
}

int wbk_selftest_bounded_wait(uint64_t timeout_ns, wbk_stream_t stream) {
  if (timeout_ns == 0 || timeout_ns > 10ull * 1000000000ull)
    return fail(WBK_ERR_INVALID_ARG, "wbk_selftest_bounded_wait: timeout must be in (0, 10 s]");
  selftest_wait_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(timeout_ns);
  return cuda_check(cudaGetLastError(), "selftest launch");
}

}  // extern "C"
