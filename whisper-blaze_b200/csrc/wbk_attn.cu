// Fused multi-head attention forward, out = softmax(Q K^T * scale) V, on B200
// tcgen05 (head dim 64, fp16 in/out, fp32 scores and accumulation).
//
// Semantics of the reference's encoder_self_attn / flash_attn_forward
// (csrc/kernels/flash_attn_hopper.cu:297-344, no causal mask, scale =
// 1/sqrt(D)), whose kernel is unfinished upstream (its own test,
// tests/test_kernels.py:297-330, is xfail against SDPA); the gate here is that
// test's: relative L2 error against fp32 SDPA. In the encoder stack this kernel
// replaces torch SDPA on the strided q/k/v views of the fused QKV output and
// also reports max|out| for the quantiser that follows.
//
// Design (one persistent CTA per SM, 384 threads):
//   * a work unit = two 128-row query tiles of one (batch, head); units are
//     dealt round-robin, consecutive CTAs take consecutive units of the same
//     head so its K/V tiles are shared through L2;
//   * warp 8: TMA producer (warps 8-11 hand registers to the softmax
//     warpgroups with setmaxnreg; 10 and 11 only take part in that). Q tiles and a 3-stage ring of K/V tiles
//     [128 keys x 64 dims], 4-D tensor maps over (dim, position, head, batch)
//     with 128-byte swizzle; rows past the sequence end read as zeros;
//   * warp 9: TMEM owner + single-thread tcgen05.mma issuer (kind::f16).
//     S_t = Q_t K^T (M128 N128, K-major operands) into TMEM; O_t += P_t V
//     (M128 N64) with P_t read from TMEM as the A operand and V as an
//     MN-major B operand. The next tile's two S products are issued before the
//     current tile's two PV products, so each softmax finds its next scores
//     ready;
//   * warps 0-3 / 4-7: one softmax warpgroup per query tile, one thread per
//     query row (its TMEM lane), with most of the CTA's registers
//     (setmaxnreg). Scores -> row max (3-input max) -> exp2 -> fp16 P written
//     to TMEM, row sum in fp32 of the fp16 P values; the running max is only
//     raised (and O rescaled in TMEM) when a tile's max exceeds it by more
//     than 2^8, so rescaling is rare. Exponentials are ex2.approx.f32 by
//     default, or ex2.approx.f16x2 (two per MUFU operation) with
//     WBK_ATTN_EXP=f16. At the end of a unit the warpgroup drains O, divides
//     by the row sum, stores fp16 rows and accumulates max|out|.
//
// Throughput (measured on B200): tcgen05.mma kind::f16 runs at the full
// 8192 FLOP/clk per SM with both operands in shared memory and N >= 128, but
// an MMA whose A operand is read from TMEM costs ~87 clocks per K=16 step
// whatever N is, and N = 64 halves the rate. With head dim 64 the PV product
// (N = 64, P from TMEM) therefore bounds this kernel at ~1900 clocks per
// pair of 128 x 128 tiles, and in practice (softmax TMEM traffic alongside)
// it runs at about half of that.
// TMEM columns: S0 [0,128) S1 [128,256) P0 [256,320) P1 [320,384)
// O0 [384,448) O1 [448,512).
//
// Every mbarrier wait is bounded (%globaltimer); a wait that runs out records
// WBK_ERR_DEVICE_TIMEOUT in this unit's device word, raises the CTA abort
// flag, and every role leaves its loop; in-flight copies and MMAs are drained
// with bounded waits before TMEM is freed.
#include <cstdlib>
#include <mutex>
#include <string>
#include <vector>

#include "wbk_common.cuh"
#include "wbk_sm100.cuh"

namespace wbk {
namespace {

constexpr int HD = 64;                  // head dim
constexpr int BQ = 128;                 // query rows per tile
constexpr int BKV = 128;                // keys per tile
constexpr int KV_STAGES = 3;
constexpr int TILE_BYTES = BQ * HD * 2;  // 16 KB per Q, K or V tile
constexpr int THREADS = 384;            // warps 0-7 softmax, 8 producer, 9 MMA, 10-11 idle
// Register split (setmaxnreg): the launch gives every thread kLaunchRegs or
// more (ptxas -v shows 168 for 384 threads); the producer/MMA warpgroup
// gives registers back and the two softmax warpgroups take them:
// 256 * kSoftmaxRegs + 128 * kControlRegs must not exceed 384 * the launch
// count, which the host checks (kMinLaunchRegs) before every first launch.
constexpr int kLaunchRegs = 168;
constexpr int kSoftmaxRegs = 208;
constexpr int kControlRegs = 80;
constexpr int kMinLaunchRegs = (256 * kSoftmaxRegs + 128 * kControlRegs + THREADS - 1) / THREADS;
constexpr uint32_t TMEM_COLS = 512;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

__device__ __forceinline__ uint32_t s_col(int t) { return static_cast<uint32_t>(t * 128); }
__device__ __forceinline__ uint32_t p_col(int t) { return static_cast<uint32_t>(256 + t * 64); }
__device__ __forceinline__ uint32_t o_col(int t) { return static_cast<uint32_t>(384 + t * 64); }

enum : uint32_t {
  ASITE_PRODUCER = 21,
  ASITE_MMA_Q = 22,
  ASITE_MMA_K = 23,
  ASITE_MMA_SFREE = 24,
  ASITE_MMA_V = 25,
  ASITE_MMA_P = 26,
  ASITE_MMA_OFREE = 27,
  ASITE_SOFTMAX_S = 28,
  ASITE_SOFTMAX_PV = 29,
  ASITE_DRAIN = 30,
};

struct AttnSmem {
  uint8_t q[2][TILE_BYTES];  // 1024-byte aligned (swizzle atoms)
  uint8_t k[KV_STAGES][TILE_BYTES];
  uint8_t v[KV_STAGES][TILE_BYTES];
  uint64_t q_full[2], q_empty[2];
  uint64_t k_full[KV_STAGES], v_full[KV_STAGES], kv_empty[KV_STAGES];
  uint64_t s_full[2], s_free[2], p_full[2], pv_done[2], o_free[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};
constexpr size_t kSmemBytes = sizeof(AttnSmem) + 1024;
static_assert(kSmemBytes <= 232448, "shared memory budget");

struct AttnParams {
  int heads, seq_q, seq_k;
  int units_per_bh;  // ceil(ceil(seq_q / 128) / 2)
  int num_units;
  int kv_tiles;
  float scale_log2;  // scale * log2(e)
  __half* out;
  int64_t o_sb, o_sh, o_ss;  // element strides of out (batch, head, position); dim stride 1
  uint32_t* out_amax;
  uint32_t idesc_s, idesc_o;
  uint64_t timeout_ns;
};

__device__ __forceinline__ void tma_load_4d(const CUtensorMap* map, uint64_t* bar, void* dst, int x, int y, int z,
                                            int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

// D[tmem] (+)= A[smem] . B[smem], 16-bit operands.
__device__ __forceinline__ void umma_f16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  const uint32_t z = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(z)
      : "memory");
}

// D[tmem] (+)= A[tmem] . B[smem], 16-bit operands; A rows are TMEM lanes, two
// K elements per 32-bit column.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  const uint32_t z = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(z)
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns from registers: thread i writes lane (base+i).
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory descriptor of an MN-major 16-bit operand tile written by TMA
// with 128-byte swizzle: each 128-byte row holds the 64 N elements of one K
// index, 8-row (1024-byte) swizzle atoms stacked along K. Fields as in
// make_sw128_desc; the stride-dimension offset (1024 B) steps between 8-K
// groups; the leading-dimension offset (between 64-wide N blocks) is unused
// for N = 64.
__device__ __forceinline__ uint64_t make_sw128_mn_desc(const void* smem_ptr) {
  const uint32_t addr = smem_u32(smem_ptr);
  uint64_t d = static_cast<uint64_t>((addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed-fp16 pieces of the softmax: two fp32 -> one f16x2 (lo in the low
// half), 2^x on both halves in one MUFU operation, and the fp32 row sum fed
// straight from fp16 operands (sm_100 mixed-precision add), so the sum is of
// exactly the fp16 P values the PV product uses.
__device__ __forceinline__ uint32_t f16x2_pack(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}
__device__ __forceinline__ uint32_t ex2_f16x2(uint32_t x) {
  uint32_t y;
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
__device__ __forceinline__ float add_f16x2_f32(uint32_t h, float acc) {
  float r;
  asm("{\n\t.reg .f16 lo, hi;\n\t.reg .f32 t;\n\tmov.b32 {lo, hi}, %1;\n\t"
      "add.f32.f16 t, lo, %2;\n\tadd.f32.f16 %0, hi, t;\n\t}"
      : "=f"(r) : "r"(h), "f"(acc));
  return r;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Bounded wait taken by a whole warp, with a warp-uniform result: every lane
// leaves together, so the .sync.aligned tcgen05 loads and stores that follow
// run on a converged warp, and a lane that saw the abort takes the others along.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          uint64_t timeout_ns, uint32_t site) {
  const bool ok = mbar_wait_inl(bar, parity, abort_flag, timeout_ns, site);
  return __all_sync(0xFFFFFFFFu, ok);
}

__device__ __forceinline__ void unit_coords(const AttnParams& p, int u, int& b, int& h, int& q0) {
  const int bh = u / p.units_per_bh;
  q0 = (u - bh * p.units_per_bh) * 2 * BQ;
  b = bh / p.heads;
  h = bh - b * p.heads;
}

// kExpF16: exponentials as ex2.approx.f16x2 on fp16 arguments (two per MUFU
// operation); otherwise ex2.approx.f32 on fp32 arguments, then rounded to fp16.
template <bool kExpF16>
__global__ void __launch_bounds__(THREADS, 1)
attn_fwd_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                const __grid_constant__ CUtensorMap tmap_v, const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  AttnSmem& s = *reinterpret_cast<AttnSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  volatile int* abort_flag = &s.abort_flag;

  if (threadIdx.x == 0) {
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s.q_full[t], 1);
      mbar_init(&s.q_empty[t], 1);
      mbar_init(&s.s_full[t], 1);
      mbar_init(&s.s_free[t], BQ);
      mbar_init(&s.p_full[t], BQ);
      mbar_init(&s.pv_done[t], 1);
      mbar_init(&s.o_free[t], BQ);
    }
    for (int i = 0; i < KV_STAGES; ++i) {
      mbar_init(&s.k_full[i], 1);
      mbar_init(&s.v_full[i], 1);
      mbar_init(&s.kv_empty[i], 1);
    }
    mbar_init(&s.drain, 1);
    s.abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_tmap(&tmap_q);
    prefetch_tmap(&tmap_k);
    prefetch_tmap(&tmap_v);
  }
  if (warp == 9) {
    tmem_alloc(&s.tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = s.tmem_base;
  const int n = p.kv_tiles;

  if (warp >= 8) {
   asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kControlRegs));
   if (warp == 8) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t g = 0;             // K/V tiles issued
      uint32_t q_loads[2] = {0, 0};  // Q tiles issued per buffer
      bool ok = true;
      for (int u = blockIdx.x; u < p.num_units && ok; u += gridDim.x) {
        int b, h, q0;
        unit_coords(p, u, b, h, q0);
        for (int t = 0; t < 2 && ok; ++t) {
          ok = mbar_wait_inl(&s.q_empty[t], (q_loads[t] & 1u) ^ 1u, abort_flag, p.timeout_ns, ASITE_PRODUCER);
          if (!ok) break;
          mbar_arrive_expect_tx(&s.q_full[t], TILE_BYTES);
          tma_load_4d(&tmap_q, &s.q_full[t], s.q[t], 0, q0 + t * BQ, h, b);
          ++q_loads[t];
        }
        for (int j = 0; j < n && ok; ++j) {
          const int st = static_cast<int>(g % KV_STAGES);
          const uint32_t ph = (g / KV_STAGES) & 1u;
          ok = mbar_wait_inl(&s.kv_empty[st], ph ^ 1u, abort_flag, p.timeout_ns, ASITE_PRODUCER);
          if (!ok) break;
          mbar_arrive_expect_tx(&s.k_full[st], TILE_BYTES);
          tma_load_4d(&tmap_k, &s.k_full[st], s.k[st], 0, j * BKV, h, b);
          mbar_arrive_expect_tx(&s.v_full[st], TILE_BYTES);
          tma_load_4d(&tmap_v, &s.v_full[st], s.v[st], 0, j * BKV, h, b);
          ++g;
        }
      }
      if (ok) {
        // Tail: every stage and Q buffer released, so no tcgen05.commit to this
        // CTA's barriers is still in flight when it exits.
        for (uint32_t i = 0, gt = g; i < KV_STAGES && ok; ++i, ++gt)
          ok = mbar_wait_inl(&s.kv_empty[gt % KV_STAGES], ((gt / KV_STAGES) & 1u) ^ 1u, abort_flag, p.timeout_ns,
                         ASITE_PRODUCER);
        for (int t = 0; t < 2 && ok; ++t)
          ok = mbar_wait_inl(&s.q_empty[t], (q_loads[t] & 1u) ^ 1u, abort_flag, p.timeout_ns, ASITE_PRODUCER);
      }
      if (!ok) {
        // Abort path: let every copy already issued land before the CTA exits
        // (a phase that completed long ago reads as complete too).
        int dummy = 0;
        for (int i = 0; i < KV_STAGES; ++i) {
          const uint32_t fills = (g + KV_STAGES - 1 - static_cast<uint32_t>(i)) / KV_STAGES;  // loads into stage i
          if (fills > 0) {
            mbar_wait_inl(&s.k_full[i], (fills - 1) & 1u, &dummy, 1000000ull, ASITE_DRAIN);
            mbar_wait_inl(&s.v_full[i], (fills - 1) & 1u, &dummy, 1000000ull, ASITE_DRAIN);
          }
        }
        for (int t = 0; t < 2; ++t)
          if (q_loads[t] > 0) mbar_wait_inl(&s.q_full[t], (q_loads[t] - 1) & 1u, &dummy, 1000000ull, ASITE_DRAIN);
      }
    }
   } else if (warp == 9) {
    // ------------------------------------------------------- MMA issuer
    if (lane == 0) {
      uint32_t g = 0, ui = 0;
      bool ok = true;
      auto issue_s = [&](int t, int st) {
        const uint64_t qd = make_sw128_desc(s.q[t]);
        const uint64_t kd = make_sw128_desc(s.k[st]);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)  // K = 16 halves = 32 bytes per MMA inside the 128-byte row
          umma_f16_ss(tmem_base + s_col(t), qd + static_cast<uint64_t>(kk * 2), kd + static_cast<uint64_t>(kk * 2),
                      p.idesc_s, kk > 0 ? 1u : 0u);
        umma_commit(&s.s_full[t]);
      };
      auto issue_pv = [&](int t, int st, bool first) {
        const uint64_t vd = make_sw128_mn_desc(s.v[st]);
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk)  // 16 keys = 8 TMEM columns of P, 2048 bytes of V per MMA
          umma_f16_ts(tmem_base + o_col(t), tmem_base + p_col(t) + static_cast<uint32_t>(kk * 8),
                      vd + static_cast<uint64_t>(kk * (2048 >> 4)), p.idesc_o, (first && kk == 0) ? 0u : 1u);
        umma_commit(&s.pv_done[t]);
      };
      for (int u = blockIdx.x; u < p.num_units && ok; u += gridDim.x, ++ui) {
        for (int t = 0; t < 2 && ok; ++t)
          ok = mbar_wait_inl(&s.q_full[t], ui & 1u, abort_flag, p.timeout_ns, ASITE_MMA_Q);
        if (!ok) break;
        // prologue: S_t of the unit's first KV tile
        {
          const int st = static_cast<int>(g % KV_STAGES);
          ok = mbar_wait_inl(&s.k_full[st], (g / KV_STAGES) & 1u, abort_flag, p.timeout_ns, ASITE_MMA_K);
          if (!ok) break;
          for (int t = 0; t < 2 && ok; ++t) {
            ok = mbar_wait_inl(&s.s_free[t], (g & 1u) ^ 1u, abort_flag, p.timeout_ns, ASITE_MMA_SFREE);
            if (!ok) break;
            tc_fence_after();
            issue_s(t, st);
          }
          if (!ok) break;
          if (n == 1) {
            umma_commit(&s.q_empty[0]);
            umma_commit(&s.q_empty[1]);
          }
        }
        for (int j = 0; j < n && ok; ++j) {
          const uint32_t gj = g + static_cast<uint32_t>(j);
          const int st = static_cast<int>(gj % KV_STAGES);
          if (j + 1 < n) {
            const uint32_t gn = gj + 1;
            const int stn = static_cast<int>(gn % KV_STAGES);
            if (!mbar_wait_inl(&s.k_full[stn], (gn / KV_STAGES) & 1u, abort_flag, p.timeout_ns, ASITE_MMA_K)) {
              ok = false;
              break;
            }
            for (int t = 0; t < 2 && ok; ++t) {
              ok = mbar_wait_inl(&s.s_free[t], gj & 1u, abort_flag, p.timeout_ns, ASITE_MMA_SFREE);
              if (!ok) break;
              tc_fence_after();
              issue_s(t, stn);
            }
            if (!ok) break;
            if (j + 2 == n) {  // the unit's last S products are issued: Q may be replaced
              umma_commit(&s.q_empty[0]);
              umma_commit(&s.q_empty[1]);
            }
          }
          if (!mbar_wait_inl(&s.v_full[st], (gj / KV_STAGES) & 1u, abort_flag, p.timeout_ns, ASITE_MMA_V)) {
            ok = false;
            break;
          }
          for (int t = 0; t < 2 && ok; ++t) {
            ok = mbar_wait_inl(&s.p_full[t], gj & 1u, abort_flag, p.timeout_ns, ASITE_MMA_P);
            if (ok && j == 0) ok = mbar_wait_inl(&s.o_free[t], (ui & 1u) ^ 1u, abort_flag, p.timeout_ns, ASITE_MMA_OFREE);
            if (!ok) break;
            tc_fence_after();
            issue_pv(t, st, j == 0);
          }
          if (!ok) break;
          umma_commit(&s.kv_empty[st]);
        }
        g += static_cast<uint32_t>(n);
      }
      if (!ok) {
        // Abort path: wait for every MMA this thread issued before TMEM is freed.
        umma_commit(&s.drain);
        int dummy = 0;
        mbar_wait_inl(&s.drain, 0, &dummy, 1000000ull, ASITE_DRAIN);
      }
    }
   }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kSoftmaxRegs));
    // --------------------------------------------------------- softmax
    const int t = warp >> 2;       // query tile of this warpgroup
    const int quarter = warp & 3;  // TMEM lanes 32*quarter ..
    const int r = quarter * 32 + lane;
    const uint32_t lane_addr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
    const float sl2 = p.scale_log2;
    const int tail = p.seq_k - (n - 1) * BKV;  // valid keys in the last tile, 1..128
    float amax = 0.0f;
    uint32_t g = 0, ui = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < p.num_units && ok; u += gridDim.x, ++ui) {
      int b, h, q0;
      unit_coords(p, u, b, h, q0);
      float m = -INFINITY;  // running max of scores * scale * log2(e)
      float l = 0.0f;       // running row sum of exp2(x - m)
      for (int j = 0; j < n; ++j) {
        const uint32_t gj = g + static_cast<uint32_t>(j);
        if (!warp_wait(&s.s_full[t], gj & 1u, abort_flag, p.timeout_ns, ASITE_SOFTMAX_S)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sr[128];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(lane_addr + s_col(t) + static_cast<uint32_t>(c * 32), sr + 32 * c);
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld_wait(sr + 32 * c);
        tc_fence_before();
        mbar_arrive(&s.s_free[t]);
        float* x = reinterpret_cast<float*>(sr);
        if (j == n - 1 && tail < BKV) {
#pragma unroll
          for (int c = 0; c < 128; ++c)
            if (c >= tail) x[c] = -INFINITY;
        }
        // Row max with 8 independent chains of 3-input max (a single chain of
        // dependent maxima would leave the issue slots idle).
        float mx8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) mx8[i] = max3f(x[i], x[8 + i], x[16 + i]);
#pragma unroll
        for (int c = 24; c < 128; c += 16)
#pragma unroll
          for (int i = 0; i < 8; ++i) mx8[i] = c + 8 + i < 128 ? max3f(mx8[i], x[c + i], x[c + 8 + i]) : fmaxf(mx8[i], x[c + i]);
        const float mx = max3f(max3f(mx8[0], mx8[1], mx8[2]), max3f(mx8[3], mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]));
        const float mt = mx * sl2;
        float alpha = 1.0f;
        if (mt > m + kRescaleThreshold) {  // always true for the first tile (m = -inf)
          alpha = ex2_approx(m - mt);      // 0 for the first tile
          m = mt;
        }
        l *= alpha;
        const bool rescale = (j > 0) && __any_sync(0xFFFFFFFFu, alpha != 1.0f);
        uint32_t pw[64];
        float rs8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const float a0 = fmaf(x[2 * c], sl2, -m), a1 = fmaf(x[2 * c + 1], sl2, -m);
          if (kExpF16) {
            pw[c] = ex2_f16x2(f16x2_pack(a0, a1));
          } else {
            pw[c] = f16x2_pack(ex2_approx(a0), ex2_approx(a1));
          }
          rs8[c & 7] = add_f16x2_f32(pw[c], rs8[c & 7]);
        }
        l += ((rs8[0] + rs8[1]) + (rs8[2] + rs8[3])) + ((rs8[4] + rs8[5]) + (rs8[6] + rs8[7]));
        if (j > 0) {
          // P_t and O_t are free once the previous tile's PV product is done.
          if (!warp_wait(&s.pv_done[t], (gj - 1) & 1u, abort_flag, p.timeout_ns, ASITE_SOFTMAX_PV)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (rescale) {
#pragma unroll 1
            for (int half = 0; half < 2; ++half) {
              uint32_t orr[32];
              const uint32_t oa = lane_addr + o_col(t) + static_cast<uint32_t>(half * 32);
              tmem_ld_32x32b_x32(oa, orr);
              tmem_ld_wait(orr);
#pragma unroll
              for (int c = 0; c < 32; ++c) orr[c] = __float_as_uint(__uint_as_float(orr[c]) * alpha);
              tmem_st_32x32b_x32(oa, orr);
            }
          }
        }
        tmem_st_32x32b_x32(lane_addr + p_col(t), pw);
        tmem_st_32x32b_x32(lane_addr + p_col(t) + 32u, pw + 32);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&s.p_full[t]);
      }
      if (!ok) break;
      // ---- unit epilogue: O_t / l -> fp16 rows
      const uint32_t glast = g + static_cast<uint32_t>(n) - 1u;
      if (!warp_wait(&s.pv_done[t], glast & 1u, abort_flag, p.timeout_ns, ASITE_SOFTMAX_PV)) break;
      tc_fence_after();
      const int row = q0 + t * BQ + r;
      const float inv = 1.0f / l;
      uint4* dst = reinterpret_cast<uint4*>(p.out + b * p.o_sb + h * p.o_sh + static_cast<int64_t>(row) * p.o_ss);
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        uint32_t orr[32];
        tmem_ld_32x32b_x32(lane_addr + o_col(t) + static_cast<uint32_t>(half * 32), orr);
        tmem_ld_wait(orr);
        if (half == 1) {  // O_t fully read: the next unit's first PV may overwrite it
          tc_fence_before();
          mbar_arrive(&s.o_free[t]);
        }
        if (row < p.seq_q) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            float o[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              o[e] = __uint_as_float(orr[8 * c + e]) * inv;
              amax = fmaxf(amax, fabsf(o[e]));
            }
            uint4 w;
            uint32_t* wp = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const __half2 hv = __floats2half2_rn(o[2 * e], o[2 * e + 1]);
              wp[e] = *reinterpret_cast<const uint32_t*>(&hv);
            }
            dst[half * 4 + c] = w;
          }
        }
      }
      g += static_cast<uint32_t>(n);
    }
    if (p.out_amax != nullptr) {
      const uint32_t bits = warp_max_u32(static_cast<uint32_t>(__half_as_ushort(__float2half_rn(amax))));
      if (lane == 0 && bits != 0u) atomicMax(p.out_amax, bits);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// 4-D tensor map over a [batch, heads, seq, 64] fp16 view with arbitrary
// (16-byte multiple) batch / head / position strides, box = 128 positions x 64 dims.
int make_tmap_bhsd(CUtensorMap* map, const void* base, int64_t batch, int64_t heads, int64_t seq, int64_t sb,
                   int64_t sh, int64_t ss) {
  auto encode = get_encode_fn();
  if (encode == nullptr) return fail(WBK_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(HD), static_cast<cuuint64_t>(seq),
                              static_cast<cuuint64_t>(heads), static_cast<cuuint64_t>(batch)};
  const cuuint64_t strides[3] = {static_cast<cuuint64_t>(ss * 2), static_cast<cuuint64_t>(sh * 2),
                                 static_cast<cuuint64_t>(sb * 2)};
  const cuuint32_t box[4] = {HD, BQ, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(WBK_ERR_CUDA, "cuTensorMapEncodeTiled (attention) failed (%d)", static_cast<int>(r));
  return WBK_OK;
}

// tcgen05 instruction descriptor, kind::f16: D fp32 (bit 4), A and B fp16
// (format 0 at bits 7 and 10), B major-ness at bit 16 (1 = MN-major),
// N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t idesc_f16(int M, int N, bool b_mn_major) {
  return (1u << 4) | (static_cast<uint32_t>(b_mn_major ? 1 : 0) << 16) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

template <bool kExpF16>
int launch_attn(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const AttnParams& p, int grid,
                cudaStream_t stream) {
  static std::mutex mu;
  static std::vector<char> configured;
  const int dev = current_device();
  if (dev < 0) return fail(WBK_ERR_CUDA, "no current CUDA device");
  {
    std::lock_guard<std::mutex> lock(mu);
    if (static_cast<int>(configured.size()) <= dev) configured.resize(dev + 1, 0);
    if (!configured[dev]) {
      cudaFuncAttributes fa;
      if (int e = cuda_check(cudaFuncGetAttributes(&fa, attn_fwd_kernel<kExpF16>), "attention function attributes"))
        return e;
      if (fa.numRegs < kMinLaunchRegs)  // the setmaxnreg split would wait for registers that do not exist
        return fail(WBK_ERR_UNSUPPORTED, "attention kernel built with %d registers per thread, needs >= %d",
                    fa.numRegs, kMinLaunchRegs);
      if (int e = cuda_check(cudaFuncSetAttribute(attn_fwd_kernel<kExpF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  static_cast<int>(kSmemBytes)),
                             "attention smem attribute"))
        return e;
      configured[dev] = 1;
    }
  }
  attn_fwd_kernel<kExpF16><<<grid, THREADS, kSmemBytes, stream>>>(tq, tk, tv, p);
  return cuda_check(cudaGetLastError(), "attention launch");
}

bool stride_ok(int64_t s) { return s > 0 && (s * 2) % 16 == 0 && (s * 2) < (int64_t(1) << 40); }

}  // namespace

int attn_read_device_error(uint32_t* v, bool clear) {
  if (int e = cuda_check(cudaMemcpyFromSymbol(v, g_device_error, sizeof(*v)), "attention device error read")) return e;
  if (clear) {
    const uint32_t zero = 0;
    if (int e = cuda_check(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero)), "attention device error clear"))
      return e;
  }
  return WBK_OK;
}

}  // namespace wbk

using namespace wbk;

extern "C" {

int wbk_attention_f16(const void* q, const void* k, const void* v, void* out, int64_t batch, int64_t heads,
                      int64_t seq_q, int64_t seq_k, int64_t head_dim, const int64_t* strides, float scale,
                      uint32_t* out_amax_bits, wbk_stream_t stream) {
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr || strides == nullptr)
    return fail(WBK_ERR_INVALID_ARG, "wbk_attention_f16: null pointer");
  if (batch < 0 || heads < 0 || seq_q < 0 || seq_k < 0)
    return fail(WBK_ERR_INVALID_ARG, "wbk_attention_f16: negative size");
  if (head_dim != HD) return fail(WBK_ERR_UNSUPPORTED, "wbk_attention_f16: head_dim %lld (only 64)", (long long)head_dim);
  if (batch == 0 || heads == 0 || seq_q == 0) return WBK_OK;
  if (seq_k == 0) return fail(WBK_ERR_INVALID_ARG, "wbk_attention_f16: seq_k = 0 with queries present");
  if (batch > (1 << 30) || heads > (1 << 30) || seq_q > (1 << 30) || seq_k > (1 << 30))
    return fail(WBK_ERR_UNSUPPORTED, "wbk_attention_f16: size exceeds 2^30");
  for (int i = 0; i < 12; ++i)
    if (!stride_ok(strides[i]))
      return fail(WBK_ERR_UNSUPPORTED, "wbk_attention_f16: stride[%d] = %lld is not a positive multiple of 8 elements",
                  i, (long long)strides[i]);
  const void* ptrs[4] = {q, k, v, out};
  for (const void* ptr : ptrs)
    if (!aligned(ptr, 16)) return fail(WBK_ERR_UNSUPPORTED, "wbk_attention_f16: pointer %p is not 16-byte aligned", ptr);
  if (out_amax_bits != nullptr && !aligned(out_amax_bits, 4))
    return fail(WBK_ERR_INVALID_ARG, "wbk_attention_f16: out_amax_bits misaligned");

  CUtensorMap tq, tk, tv;
  if (int e = make_tmap_bhsd(&tq, q, batch, heads, seq_q, strides[0], strides[1], strides[2])) return e;
  if (int e = make_tmap_bhsd(&tk, k, batch, heads, seq_k, strides[3], strides[4], strides[5])) return e;
  if (int e = make_tmap_bhsd(&tv, v, batch, heads, seq_k, strides[6], strides[7], strides[8])) return e;

  AttnParams p{};
  p.heads = static_cast<int>(heads);
  p.seq_q = static_cast<int>(seq_q);
  p.seq_k = static_cast<int>(seq_k);
  const int64_t q_tiles = (seq_q + BQ - 1) / BQ;
  p.units_per_bh = static_cast<int>((q_tiles + 1) / 2);
  const int64_t units = batch * heads * p.units_per_bh;
  if (units > (int64_t(1) << 31) - 1) return fail(WBK_ERR_UNSUPPORTED, "wbk_attention_f16: too many work units");
  p.num_units = static_cast<int>(units);
  p.kv_tiles = static_cast<int>((seq_k + BKV - 1) / BKV);
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = static_cast<__half*>(out);
  p.o_sb = strides[9];
  p.o_sh = strides[10];
  p.o_ss = strides[11];
  p.out_amax = out_amax_bits;
  p.idesc_s = idesc_f16(BQ, BKV, false);
  p.idesc_o = idesc_f16(BQ, HD, true);
  p.timeout_ns = wait_timeout_ns();

  static const bool exp_f16 = [] {
    const char* e = std::getenv("WBK_ATTN_EXP");
    return e != nullptr && std::string(e) == "f16";
  }();
  const int sms = sm_count() > 0 ? sm_count() : 148;
  const int grid = p.num_units < sms ? p.num_units : sms;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  return exp_f16 ? launch_attn<true>(tq, tk, tv, p, grid, st) : launch_attn<false>(tq, tk, tv, p, grid, st);
}

}  // extern "C"
