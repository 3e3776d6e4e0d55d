// FlashAttention-2 forward on sm_100a: TMA + tcgen05 MMA with TMEM accumulators.
//
// Reference: the kernel its emitter builds for examples/flash_attention.py:26-79 — per
// (batch, head, 64-row query tile): S = Q K^T, online softmax in base 2 with
// scale = log2(e)/sqrt(d) (:23), causal fill -1e30 (:56-62), P cast to fp16 before P V
// (:74-75), O /= l at the end (:77-78); sm_80 mma.sync with smem round trips for the row
// statistics (codegen.py:972-984, :1062-1073).
//
// Design: one CTA = one (batch, head, 256-query block) = two 128-row query tiles that
// share every K/V tile (384 threads, 12 warps = 3 warpgroups).  Causal attention runs the same
// units on a persistent grid (fa2_persist_kernel, further down) when they fill its rounds:
//   warps 0-3   softmax, O rescale and the O / l -> fp16 epilogue of query tile 0: one thread
//               per query row (its TMEM lane), the row's 128 scores in registers
//   warps 4-7   the same for query tile 1
//   warp 8      TMEM owner (512 columns: S0, S1, O0, O1) and MMA issuer
//   warp 9      TMA: Q0, Q1 once, then K_j and V_j (2-stage rings each) with K running one
//               tile ahead; 3-D tensor maps [B*H, S, D] zero-fill rows past S and never
//               cross heads
//   warps 10-11 idle (they complete warpgroup 2 for the register split)
// Registers: launched at 168 per thread; warpgroup 2 gives up registers down to 72 and the
// two softmax warpgroups take them, up to 216 (setmaxnreg), so a softmax thread holds its
// row's scores, exponentials and packed P without spilling.
// Per KV tile j the MMA warp issues, per query tile i: O_i += P_i V_j (A = P_i from TMEM,
// fp16 pairs packed over the first 64 S_i columns; B = V_j N-major in smem) and then
// S_i = Q_i K_{j+1}^T (both operands K-major in smem), so the tensor core works on one tile
// while the other tile's softmax runs.  The softmax warps signal the low-key half of P as
// soon as it is in TMEM, and the MMA warp starts P V on those keys while the high half is
// computed; the MMA warp checks V_j and K_{j+1} before it waits for the softmax, and spins
// (bounded, never suspended) on the softmax hand-offs.  Softmax uses a lazily updated row max: O and l are
// rescaled only when the max grows by more than 2^8 (P stays <= 256, exact in the final
// O / l).  S_i of tile j is issued after P_i V_{j-1}, so once S_i is ready O_i is stable and
// the softmax warps rescale it in place without another hand-off.  Masked scores (causal
// key > query, keys >= S) contribute exactly 0, like the reference's -1e30 fill.  Every
// mbarrier wait is bounded; a wait that gives up records a status code, drains in-flight
// copies and MMAs, frees TMEM and returns.
#include <atomic>
#include <mutex>

#include "ntl_common.cuh"

namespace {

__device__ uint32_t g_fa2_status;

constexpr int BM = 128;        // rows per query tile
constexpr int QTILES = 2;      // query tiles per CTA
constexpr int BQ = BM * QTILES;
constexpr int BN = 128;        // keys per KV tile
constexpr int KSTAGES = 2, VSTAGES = 2;
constexpr int THREADS = 384;  // 3 warpgroups: softmax tile 0, softmax tile 1, MMA + TMA (+2 idle)
constexpr int REGS_LAUNCH = 168, REGS_SOFTMAX = 216, REGS_OTHER = 72;
static_assert(8 * REGS_SOFTMAX + 4 * REGS_OTHER == 12 * REGS_LAUNCH, "register split must match the launch");
static_assert(2 * REGS_SOFTMAX + REGS_OTHER <= 512, "per-SMSP register file");
constexpr int MMA_WARP = 8, TMA_WARP = 9;
constexpr int SM_WARPS_PER_TILE = 4;  // one thread per query row
constexpr uint32_t TMEM_COLS = 512;
constexpr float kRescaleLog2 = 8.0f;  // lazy-rescale threshold (log2 units)
constexpr double kPersistMinFill = 0.95;  // causal: the persistent grid's least fill of its rounds

struct Fa2Params {
  __half* o;
  int S, n_qb;
  int BH;  // batch * heads
  int causal;
  float c;          // softmax scale in log2 units
  int succ_stride;  // CTAs resident at once: block b + succ_stride is likely to start when b ends
  int64_t wait_limit;
};

struct __align__(16) Fa2Ctl {
  uint64_t q_full[QTILES];
  uint64_t k_full[KSTAGES], k_empty[KSTAGES], v_full[VSTAGES], v_empty[VSTAGES];
  uint64_t s_full[QTILES];
  uint64_t sm_done[QTILES];
  uint64_t p_lo[QTILES];     // the low-key half of P_i is in TMEM (8 warps)
  uint64_t o_final[QTILES];
  uint64_t o_staged[QTILES];  // O_i / l is in shared memory (4 warps)
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

template <int D>
struct Fa2Smem {
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + QTILES * Q_BYTES;
  static constexpr int V_OFF = K_OFF + KSTAGES * KV_BYTES;
  static constexpr int CTL_OFF = V_OFF + VSTAGES * KV_BYTES;
  static constexpr int USED = CTL_OFF + static_cast<int>(sizeof(Fa2Ctl));
  // >= 116 KB keeps one CTA per SM, so the 512-column TMEM allocation never contends.
  static constexpr int BYTES = (USED + 1024 > 118784 ? USED + 1024 : 118784);
  __host__ __device__ static constexpr uint32_t S_COL(int i) { return static_cast<uint32_t>(i * BN); }
  __host__ __device__ static constexpr uint32_t O_COL(int i) { return static_cast<uint32_t>(2 * BN + i * D); }
};

__device__ __forceinline__ void fa2_abort(Fa2Ctl* ctl, uint32_t code) {
  atomicCAS(&g_fa2_status, 0u, code);
  *reinterpret_cast<volatile int*>(&ctl->abort) = 1;
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// 2^x on the FMA pipe, for x <= ~8 (softmax exponents): x = n + f with n = round(x) via
// the 1.5*2^23 rounding constant, 2^f on [-1/2, 1/2] by a cubic fitted here for minimum
// relative error (max 7.6e-5, below fp16's half-ulp 2.4e-4 that P is rounded to), and
// 2^n added to the exponent bits.  x is clamped at -126 so the exponent never underflows;
// such terms (masked or tiny scores) become ~1e-38, i.e. 0 in fp16 P.  Used for a fixed
// quarter of the exponentials so the MUFU ex2 unit and the FMA pipe share the load.
// Two values per call, with f32x2 arithmetic.  The method is additive range reduction
// (W. J. Cody and W. Waite, "Software Manual for the Elementary Functions", 1980) with the
// result's exponent written straight into the float's bits (N. N. Schraudolph, "A Fast,
// Compact Approximation of the Exponential Function", Neural Computation 11(4), 1999); the
// cubic's coefficients were fitted for this kernel.
__device__ __forceinline__ void exp2_fma2(uint64_t x2, float& p0, float& p1) {
  constexpr float kRound = 12582912.0f;
  float x0, x1;
  f2_split(x2, x0, x1);
  x2 = f2_make(fmaxf(x0, -126.0f), fmaxf(x1, -126.0f));
  const uint64_t round2 = f2_make(kRound, kRound);
  const uint64_t t2 = f2_add(x2, round2);
  const uint64_t f2 = f2_sub(x2, f2_sub(t2, round2));
  uint64_t q2 = f2_fma(f2_make(0.055170975625514984f, 0.055170975625514984f), f2,
                       f2_make(0.24260970950126648f, 0.24260970950126648f));
  q2 = f2_fma(q2, f2, f2_make(0.6932609677314758f, 0.6932609677314758f));
  q2 = f2_fma(q2, f2, f2_make(0.9999281764030457f, 0.9999281764030457f));
  float q0, q1, t0, t1;
  f2_split(q2, q0, q1);
  f2_split(t2, t0, t1);
  p0 = __uint_as_float(__float_as_uint(q0) + (__float_as_uint(t0) << 23));
  p1 = __uint_as_float(__float_as_uint(q1) + (__float_as_uint(t1) << 23));
}

// Number of KV tiles query tile i of block qb needs (0 when the tile is past S).
__device__ __forceinline__ int kv_tiles(const Fa2Params& p, int q0_tile) {
  if (q0_tile >= p.S) return 0;
  const int all = (p.S + BN - 1) / BN;
  return p.causal ? min(all, (q0_tile + BM - 1) / BN + 1) : all;
}

// Block order (one CTA per (batch, head, 256-query block), a 1-D grid the hardware hands
// out in index order as SMs free up).  Non-causal blocks all cost the same and go by head,
// so the CTAs in flight cover ~148/n_qb heads whose K and V stay in L2.  Causal blocks go by
// groups of kCausalGroup heads, heaviest query block first within a group (the last query
// block needs every KV tile), so the blocks left at the end of the grid are the light ones:
// on [8, 32, 4096] that balances the SMs to ~99% of the mean load against ~96% for
// head-major order, and a group's K and V (2 MB per head) still fit in L2.
constexpr int kCausalGroup = 16;

__device__ __forceinline__ void decode_block(const Fa2Params& p, int w, int& qb, int& bh) {
  if (!p.causal) {
    qb = w % p.n_qb;
    bh = w / p.n_qb;
    return;
  }
  const int g0 = (w / (kCausalGroup * p.n_qb)) * kCausalGroup;  // first head of the group
  const int gs = min(kCausalGroup, p.BH - g0);
  const int within = w - g0 * p.n_qb;
  qb = p.n_qb - 1 - within / gs;
  bh = g0 + within % gs;
}

template <int D>
__global__ void __launch_bounds__(THREADS, 1) fa2_fwd_kernel(const __grid_constant__ CUtensorMap tq,
                                                             const __grid_constant__ CUtensorMap tk,
                                                             const __grid_constant__ CUtensorMap tv,
                                                             const __grid_constant__ CUtensorMap to,
                                                             const Fa2Params p) {
  using L = Fa2Smem<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Fa2Ctl* ctl = reinterpret_cast<Fa2Ctl*>(smem + L::CTL_OFF);
  volatile int* abort_flag = &ctl->abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int qb, bh;
  decode_block(p, static_cast<int>(blockIdx.x), qb, bh);
  const int q0 = qb * BQ;
  int n_t[QTILES];
#pragma unroll
  for (int i = 0; i < QTILES; ++i) n_t[i] = kv_tiles(p, q0 + i * BM);
  const int n_max = max(n_t[0], n_t[1]);

  if (warp == TMA_WARP && lane == 0) {
    // The load pipeline's barriers are set up by the thread that issues the loads, which
    // starts Q_0, K_0 and Q_1 before the CTA-wide sync (a fresh K stage needs no empty
    // wait), so the first QK^T's operands arrive during setup.  Then it prefetches into
    // L2 the Q tiles of block b + succ_stride, which the hardware hands out in index order
    // as CTAs retire: Q is read once per block, and without it the next block's first
    // load on some SM would come from DRAM.
    for (int i = 0; i < QTILES; ++i) mbar_init(&ctl->q_full[i], 1);
    for (int s = 0; s < KSTAGES; ++s) {
      mbar_init(&ctl->k_full[s], 1);
      mbar_init(&ctl->k_empty[s], 1);
    }
    for (int s = 0; s < VSTAGES; ++s) {
      mbar_init(&ctl->v_full[s], 1);
      mbar_init(&ctl->v_empty[s], 1);
    }
    fence_mbar_init();
    prefetch_tensormap(&tq);
    prefetch_tensormap(&tk);
    auto load_q = [&](int i) {
      mbar_arrive_expect_tx(&ctl->q_full[i], L::Q_BYTES);
#pragma unroll
      for (int d = 0; d < D / 64; ++d)
        tma_load_3d(smem + L::Q_OFF + i * L::Q_BYTES + d * (BM * 128), &tq, &ctl->q_full[i], d * 64, q0 + i * BM, bh);
    };
    load_q(0);
    mbar_arrive_expect_tx(&ctl->k_full[0], L::KV_BYTES);  // n_t[0] >= 1: q0 < S
#pragma unroll
    for (int d = 0; d < D / 64; ++d)
      tma_load_3d(smem + L::K_OFF + d * (BN * 128), &tk, &ctl->k_full[0], d * 64, 0, bh);
    load_q(1);
    const int64_t succ = static_cast<int64_t>(blockIdx.x) + p.succ_stride;
    if (p.succ_stride > 0 && succ < static_cast<int64_t>(gridDim.x)) {
      int qb2, bh2;
      decode_block(p, static_cast<int>(succ), qb2, bh2);
#pragma unroll
      for (int i = 0; i < QTILES; ++i)
        if (qb2 * BQ + i * BM < p.S)
#pragma unroll
          for (int d = 0; d < D / 64; ++d) tma_prefetch_3d(&tq, d * 64, qb2 * BQ + i * BM, bh2);
    }
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < QTILES; ++i) {
      mbar_init(&ctl->s_full[i], 1);
      mbar_init(&ctl->sm_done[i], SM_WARPS_PER_TILE);
      mbar_init(&ctl->p_lo[i], SM_WARPS_PER_TILE);
      mbar_init(&ctl->o_final[i], 1);
      mbar_init(&ctl->o_staged[i], SM_WARPS_PER_TILE);
    }
    mbar_init(&ctl->drain, 1);
    ctl->abort = 0;
    fence_mbar_init();
    prefetch_tensormap(&tv);
    prefetch_tensormap(&to);
  }
  if (warp == MMA_WARP) {
    tmem_alloc(&ctl->tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  if (warp >= 8) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(REGS_OTHER) : "memory");
  if (warp == TMA_WARP) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      bool ok = true;
      // Q_0, K_0, Q_1 went out before the sync.  Issue order K0, K1, V0, K2, V1, ...: K runs
      // one tile ahead of V.
      int k_issued = 1, v_issued = 0;
      auto load_k = [&](int j) -> bool {
        const int s = j % KSTAGES;
        if (!mbar_wait_bounded(&ctl->k_empty[s], ((j / KSTAGES) & 1) ^ 1, p.wait_limit, abort_flag)) return false;
        mbar_arrive_expect_tx(&ctl->k_full[s], L::KV_BYTES);
#pragma unroll
        for (int d = 0; d < D / 64; ++d)
          tma_load_3d(smem + L::K_OFF + s * L::KV_BYTES + d * (BN * 128), &tk, &ctl->k_full[s], d * 64, j * BN, bh);
        ++k_issued;
        return true;
      };
      auto load_v = [&](int j) -> bool {
        const int s = j % VSTAGES;
        if (!mbar_wait_bounded(&ctl->v_empty[s], ((j / VSTAGES) & 1) ^ 1, p.wait_limit, abort_flag)) return false;
        mbar_arrive_expect_tx(&ctl->v_full[s], L::KV_BYTES);
#pragma unroll
        for (int d = 0; d < D / 64; ++d)
          tma_load_3d(smem + L::V_OFF + s * L::KV_BYTES + d * (BN * 128), &tv, &ctl->v_full[s], d * 64, j * BN, bh);
        ++v_issued;
        return true;
      };
      for (int j = 0; j < n_max && ok; ++j) {
        if (j + 1 < n_max && !load_k(j + 1)) ok = false;
        else if (!load_v(j)) ok = false;
      }
      if (!ok && !*abort_flag) fa2_abort(ctl, NTL_STATUS_TMA_EMPTY_WAIT);
      if (!ok) {
        // Drain every copy this thread issued before the CTA exits.
        for (int i = 0; i < QTILES; ++i)
          if (!mbar_wait_bounded(&ctl->q_full[i], 0, int64_t(1) << 24, nullptr))
            atomicCAS(&g_fa2_status, 0u, NTL_STATUS_DRAIN_WAIT);
        for (int j = max(0, k_issued - KSTAGES); j < k_issued; ++j)
          if (!mbar_wait_bounded(&ctl->k_full[j % KSTAGES], (j / KSTAGES) & 1, int64_t(1) << 24, nullptr))
            atomicCAS(&g_fa2_status, 0u, NTL_STATUS_DRAIN_WAIT);
        for (int j = max(0, v_issued - VSTAGES); j < v_issued; ++j)
          if (!mbar_wait_bounded(&ctl->v_full[j % VSTAGES], (j / VSTAGES) & 1, int64_t(1) << 24, nullptr))
            atomicCAS(&g_fa2_status, 0u, NTL_STATUS_DRAIN_WAIT);
      }
    }
  } else if (warp == MMA_WARP) {
    // ------------------------------------------------------------------ MMA issuer
    if (elect_one_lane()) {
      constexpr uint32_t idesc_s = umma_idesc_f16_f32(BM, BN, 0, 0);  // B = K tile, K-major
      constexpr uint32_t idesc_o = umma_idesc_f16_f32(BM, D, 0, 1);   // B = V tile, N-major
      bool ok = true;
      auto spin_or_abort = [&](uint64_t* bar, uint32_t parity) -> bool {
        if (mbar_spin_bounded(bar, parity, p.wait_limit, abort_flag)) return true;
        if (!*abort_flag) fa2_abort(ctl, NTL_STATUS_MMA_FULL_WAIT);
        return false;
      };
      auto wait_or_abort = [&](uint64_t* bar, uint32_t parity) -> bool {
        if (mbar_wait_bounded(bar, parity, p.wait_limit, abort_flag)) return true;
        if (!*abort_flag) fa2_abort(ctl, NTL_STATUS_MMA_FULL_WAIT);
        return false;
      };
      auto issue_s = [&](int i, int j) {  // S_i = Q_i K_j^T
        const uint32_t q_addr = smem_u32(smem + L::Q_OFF + i * L::Q_BYTES);
        const uint32_t k_addr = smem_u32(smem + L::K_OFF + (j % KSTAGES) * L::KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
          tc_mma_f16_ss(tmem + L::S_COL(i), umma_desc_sw128(q_addr + off, 16, 1024),
                        umma_desc_sw128(k_addr + off, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
        }
        tc_commit(&ctl->s_full[i]);
      };
      if (wait_or_abort(&ctl->k_full[0], 0)) {
        // Every issued load is waited for, a dead query tile's (all rows past S) included, so
        // the CTA never exits with a copy into its shared memory in flight.
        for (int i = 0; i < QTILES && ok; ++i) {
          if (!wait_or_abort(&ctl->q_full[i], 0)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (n_t[i] > 0) issue_s(i, 0);
        }
        if (ok) tc_commit(&ctl->k_empty[0]);  // K_0 is free once both QK^T retire
      } else {
        ok = false;
      }
      for (int j = 0; j < n_max && ok; ++j) {
        const int s = j % VSTAGES;
        for (int i = 0; i < QTILES && ok; ++i) {
          if (j >= n_t[i]) continue;
          // V_j and K_{j+1} were loaded long before the softmax finishes: check them first,
          // so that only the softmax hand-off is on the critical path.
          if (!wait_or_abort(&ctl->v_full[s], (j / VSTAGES) & 1)) {
            ok = false;
            break;
          }
          if (j + 1 < n_t[i] && !wait_or_abort(&ctl->k_full[(j + 1) % KSTAGES], ((j + 1) / KSTAGES) & 1)) {
            ok = false;
            break;
          }
          if (!spin_or_abort(&ctl->p_lo[i], j & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t v_addr = smem_u32(smem + L::V_OFF + s * L::KV_BYTES);
#pragma unroll
          for (int kk = 0; kk < BN / 32; ++kk)  // keys [0, 64): packed S columns [0, 32)
            tc_mma_f16_ts(tmem + L::O_COL(i), tmem + L::S_COL(i) + kk * 8,
                          umma_desc_sw128(v_addr + kk * 2048, BN * 128, 1024), idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
          if (!spin_or_abort(&ctl->sm_done[i], j & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = BN / 32; kk < BN / 16; ++kk)  // keys [64, 128): packed S columns [32, 64)
            tc_mma_f16_ts(tmem + L::O_COL(i), tmem + L::S_COL(i) + kk * 8,
                          umma_desc_sw128(v_addr + kk * 2048, BN * 128, 1024), idesc_o, 1u);
          if (j == n_t[i] - 1) tc_commit(&ctl->o_final[i]);
          if (j + 1 < n_t[i]) issue_s(i, j + 1);
        }
        if (ok) {
          tc_commit(&ctl->v_empty[s]);                                    // V_j consumed by both P V
          if (j + 1 < n_max) tc_commit(&ctl->k_empty[(j + 1) % KSTAGES]);  // K_{j+1} by both QK^T
        }
      }
      if (!ok) {
        tc_commit(&ctl->drain);
        if (!mbar_wait_bounded(&ctl->drain, 0, int64_t(1) << 24, nullptr))
          atomicCAS(&g_fa2_status, 0u, NTL_STATUS_DRAIN_WAIT);
      }
    }
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(REGS_SOFTMAX) : "memory");
    // ------------------------------------------------------------------ softmax warps
    // Warp w: query tile i = w/4; thread = row r = 32*(w%4) + lane = its TMEM lane (the lanes a
    // warp may access), all BN keys of the row in registers: row max and sum need no exchange.
    const int i = warp >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int tile_q0 = q0 + i * BM;
    const int qrow = tile_q0 + r;
    const int n_mine = kv_tiles(p, tile_q0);
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_addr = tmem + lane_off + L::S_COL(i);
    const uint32_t o_addr = tmem + lane_off + L::O_COL(i);
    const float c = p.c;
    const int key_lim = p.causal ? min(p.S, qrow + 1) : p.S;  // keys < key_lim are kept
    float m_use = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < n_mine; ++j) {
      if (!mbar_wait_bounded(&ctl->s_full[i], j & 1, p.wait_limit, abort_flag)) {
        if (!*abort_flag) fa2_abort(ctl, NTL_STATUS_SOFTMAX_WAIT);
        ok = false;
        break;
      }
      __syncwarp();
      tc_fence_after();
      uint32_t sv[BN];  // S[r, j*BN + k]
#pragma unroll
      for (int ch = 0; ch < BN / 32; ++ch)
        tmem_ld_32x32b_x32(s_addr + ch * 32, *reinterpret_cast<uint32_t(*)[32]>(sv + ch * 32));
      tc_wait_ld();
      if ((j * BN + BN > p.S) || (p.causal && j * BN + BN - 1 > tile_q0)) {
#pragma unroll
        for (int k = 0; k < BN; ++k)
          if (j * BN + k >= key_lim) sv[k] = __float_as_uint(-INFINITY);
      }
      float mx;
      {
        float x[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int k = 0; k < BN; k += 8) {
          x[0] = fmax3(x[0], __uint_as_float(sv[k]), __uint_as_float(sv[k + 1]));
          x[1] = fmax3(x[1], __uint_as_float(sv[k + 2]), __uint_as_float(sv[k + 3]));
          x[2] = fmax3(x[2], __uint_as_float(sv[k + 4]), __uint_as_float(sv[k + 5]));
          x[3] = fmax3(x[3], __uint_as_float(sv[k + 6]), __uint_as_float(sv[k + 7]));
        }
        mx = fmax3(fmaxf(x[0], x[1]), x[2], x[3]);
      }
      // lazy max
      float rs = 1.0f;
      bool moved = false;
      if (j == 0) {
        m_use = mx;
      } else if ((mx - m_use) * c > kRescaleLog2) {
        rs = ex2_approx((m_use - mx) * c);
        m_use = mx;
        moved = true;
      }
      if (__any_sync(0xffffffffu, moved)) {
        // O_i = P_{<j} V is complete: S_i of this tile was issued after the last P_i V.
#pragma unroll 1
        for (int ch = 0; ch < D / 32; ++ch) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(o_addr + ch * 32, o);
          tc_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * rs);
          tmem_st_32x32b_x32(o_addr + ch * 32, o);
        }
      }
      // p = exp2(s*c - m*c) -> fp16 pairs: keys 2u, 2u+1 in S column u (columns already read)
      const uint64_t c2 = f2_make(c, c);
      const uint64_t nm2 = f2_make(-m_use * c, -m_use * c);
      uint64_t acc2[2] = {0ull, 0ull};
#pragma unroll
      for (int ch = 0; ch < BN / 32; ++ch) {
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int k = ch * 32 + 2 * e;
          const uint64_t x2 = f2_fma(f2_make(__uint_as_float(sv[k]), __uint_as_float(sv[k + 1])), c2, nm2);
          float p0, p1;
          if ((e & 3) == 3) {  // one pair in four on the FMA pipe
            exp2_fma2(x2, p0, p1);
          } else {
            float x0, x1;
            f2_split(x2, x0, x1);
            p0 = ex2_approx(x0);
            p1 = ex2_approx(x1);
          }
          acc2[e & 1] = f2_add(acc2[e & 1], f2_make(p0, p1));
          pk[e] = pack_half2(p0, p1);
        }
        tmem_st_32x32b_x16(s_addr + ch * 16, pk);
        if (ch == BN / 64 - 1) {
          // keys [0, BN/2) of P are in TMEM: the MMA warp may start on them
          tc_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&ctl->p_lo[i]);
        }
      }
      float sum;
      {
        float u0, u1;
        f2_split(f2_add(acc2[0], acc2[1]), u0, u1);
        sum = u0 + u1;
      }
      l = (j == 0) ? sum : __fmaf_rn(l, rs, sum);
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->sm_done[i]);
    }
    // epilogue: O / l -> fp16.  Each thread writes its row into Q_i's shared buffer (free:
    // Q_i's last QK^T retired before o_final) in the layout the 128-byte-swizzled Q tiles
    // have, and one thread stores the tile with one TMA store per 64-column box; the tensor
    // map clips rows past S.
    if (ok && n_mine > 0) {
      if (!mbar_wait_bounded(&ctl->o_final[i], 0, p.wait_limit, abort_flag)) {
        if (!*abort_flag) fa2_abort(ctl, NTL_STATUS_SOFTMAX_WAIT);
      } else {
        __syncwarp();
        tc_fence_after();
        const float inv_l = 1.0f / l;
        uint32_t ov[D];  // the row of O: every chunk in flight before one wait
#pragma unroll
        for (int ch = 0; ch < D / 32; ++ch)
          tmem_ld_32x32b_x32(o_addr + ch * 32, *reinterpret_cast<uint32_t(*)[32]>(ov + ch * 32));
        tc_wait_ld();
        uint8_t* ot = smem + L::Q_OFF + i * L::Q_BYTES;
#pragma unroll
        for (int ch = 0; ch < D / 32; ++ch) {
          uint32_t hv[16];
#pragma unroll
          for (int e = 0; e < 16; ++e)
            hv[e] = pack_half2(__uint_as_float(ov[ch * 32 + 2 * e]) * inv_l,
                               __uint_as_float(ov[ch * 32 + 2 * e + 1]) * inv_l);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const int u = ch * 4 + q4;  // 16-byte unit of the row; 8 units per 64-column box
            uint8_t* dst = ot + (u >> 3) * (BM * 128) + r * 128 + (((u & 7) ^ (r & 7)) << 4);
            *reinterpret_cast<uint4*>(dst) = make_uint4(hv[4 * q4], hv[4 * q4 + 1], hv[4 * q4 + 2], hv[4 * q4 + 3]);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->o_staged[i]);
        if (quarter == 0 && lane == 0) {
          if (mbar_wait_bounded(&ctl->o_staged[i], 0, p.wait_limit, abort_flag)) {
#pragma unroll
            for (int d = 0; d < D / 64; ++d) tma_store_3d(&to, ot + d * (BM * 128), d * 64, tile_q0, bh);
            bulk_commit();
            bulk_wait_read();
          } else if (!*abort_flag) {
            fa2_abort(ctl, NTL_STATUS_SOFTMAX_WAIT);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == MMA_WARP) tmem_dealloc(tmem, TMEM_COLS);
}


// ===================================================================== persistent grid (causal)
//
// The same units, KV steps and softmax as fa2_fwd_kernel above, on a persistent grid of one CTA
// per SM: each CTA runs a fixed sequence of units back to back, so the next unit's Q and first
// K/V tiles load, and its first QK^T runs, while the current unit's last P V and epilogue finish.
// Causal units are short (half of them need fewer than half the KV tiles), so the per-unit start
// and end this overlaps are a large share of their time: +3% causal on [8, 32, 4096, 128]
// (bit-identical output).  Non-causal measured 2-4% slower persistent (each KV step of the longer
// loop ran ~7% slower by clock64 trace), so it keeps fa2_fwd_kernel.  The per-step code is a copy
// of fa2_fwd_kernel's rather than a shared function: factoring the two kernels' softmax and MMA
// steps into common device functions made fa2_fwd_kernel 2.5-5% slower (same output).
//
// Differences from fa2_fwd_kernel: barrier phases run on per-tile step counters across units;
// the K and V rings run one sequence across units; Q_i of the next unit loads once the last
// QK^T of tile i retired (q_empty); O / l leaves through a dedicated staging tile that the two
// query tiles take in turn (ostage_free), so the next unit's Q can load meanwhile; the register
// split is 200 / 104 (the MMA and TMA threads carry loop state across units: at 216 / 72 they
// spilled).  O_i's TMEM is reused by the next unit only after the softmax warps, which wrote its
// epilogue, hand off that unit's first P.
constexpr int PER_REGS_SOFTMAX = 200, PER_REGS_OTHER = 104;
static_assert(8 * PER_REGS_SOFTMAX + 4 * PER_REGS_OTHER == 12 * REGS_LAUNCH, "register split must match the launch");
static_assert(2 * PER_REGS_SOFTMAX + PER_REGS_OTHER <= 512, "per-SMSP register file");

struct PersistParams {
  int S, n_qb;
  int BH;  // batch * heads
  int units;  // n_qb * BH
  int causal;
  float c;          // softmax scale in log2 units
  int64_t wait_limit;
};

struct __align__(16) PersistCtl {
  uint64_t q_full[QTILES], q_empty[QTILES];
  uint64_t k_full[KSTAGES], k_empty[KSTAGES], v_full[VSTAGES], v_empty[VSTAGES];
  uint64_t s_full[QTILES];
  uint64_t sm_done[QTILES];
  uint64_t p_lo[QTILES];     // the low-key half of P_i is in TMEM (4 warps)
  uint64_t o_final[QTILES];
  uint64_t o_staged[QTILES];  // O_i / l is in the staging buffer (4 warps)
  uint64_t ostage_free;       // the staging buffer has been read out by the last TMA store
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

template <int D>
struct PersistSmem {
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + QTILES * Q_BYTES;
  static constexpr int V_OFF = K_OFF + KSTAGES * KV_BYTES;
  static constexpr int OS_OFF = V_OFF + VSTAGES * KV_BYTES;  // O staging, one 128-row tile
  static constexpr int CTL_OFF = OS_OFF + Q_BYTES;
  static constexpr int USED = CTL_OFF + static_cast<int>(sizeof(PersistCtl));
  // >= 116 KB keeps one CTA per SM, so the 512-column TMEM allocation never contends.
  static constexpr int BYTES = (USED + 1024 > 118784 ? USED + 1024 : 118784);
  static_assert(BYTES <= 232448, "shared memory per CTA");
  __host__ __device__ static constexpr uint32_t S_COL(int i) { return static_cast<uint32_t>(i * BN); }
  __host__ __device__ static constexpr uint32_t O_COL(int i) { return static_cast<uint32_t>(2 * BN + i * D); }
};

// Number of KV tiles query tile q0_tile needs (0 when the tile is past S); as kv_tiles above.
__device__ __forceinline__ int kv_tiles(const PersistParams& p, int q0_tile) {
  if (q0_tile >= p.S) return 0;
  const int all = (p.S + BN - 1) / BN;
  return p.causal ? min(all, (q0_tile + BM - 1) / BN + 1) : all;
}

__device__ __forceinline__ void fa2_abort(PersistCtl* ctl, uint32_t code) {
  atomicCAS(&g_fa2_status, 0u, code);
  *reinterpret_cast<volatile int*>(&ctl->abort) = 1;
}

// Unit order.  Within each (batch, head) the query blocks alternate heaviest and lightest:
// n_qb-1, 0, n_qb-2, 1, ... (under causal masking block qb needs about 2qb+2 KV steps), so
// consecutive units form pairs of equal total cost.  CTA c of G takes pairs c, c+G, c+2G, ...,
// both units of a pair back to back: on [8, 32, 4096] causal that puts every CTA within ~1%
// of the mean load (handing out single units round-robin: 6%), without a shared counter.  The
// G CTAs in flight cover ~G/(n_qb/2) heads, whose K and V (2 MB per head) stay in L2.
__device__ __forceinline__ void decode_unit(const PersistParams& p, int w, int& qb, int& bh) {
  bh = w / p.n_qb;
  const int k = w - bh * p.n_qb;
  qb = (k & 1) ? (k >> 1) : (p.n_qb - 1 - (k >> 1));
}

// The u-th unit (u = 0, 1, ...) of this CTA; false past the end of the sequence.
__device__ __forceinline__ bool cta_unit(const PersistParams& p, int u, int& w) {
  const int64_t pair = static_cast<int64_t>(blockIdx.x) + static_cast<int64_t>(u >> 1) * gridDim.x;
  const int64_t ww = pair * 2 + (u & 1);
  if (ww >= p.units) return false;
  w = static_cast<int>(ww);
  return true;
}

template <int D>
__global__ void __launch_bounds__(THREADS, 1) fa2_persist_kernel(const __grid_constant__ CUtensorMap tq,
                                                             const __grid_constant__ CUtensorMap tk,
                                                             const __grid_constant__ CUtensorMap tv,
                                                             const __grid_constant__ CUtensorMap to,
                                                             const PersistParams p) {
  using L = PersistSmem<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  PersistCtl* ctl = reinterpret_cast<PersistCtl*>(smem + L::CTL_OFF);
  volatile int* abort_flag = &ctl->abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (warp == TMA_WARP && lane == 0) {
    // The load pipeline's barriers are set up by the thread that issues the loads, which
    // starts the first unit's Q_0, K_0 and Q_1 before the CTA-wide sync (fresh buffers need
    // no empty wait), so the first QK^T's operands arrive during setup.  The grid never has
    // more CTAs than pairs of units, so every CTA has a first unit.
    for (int i = 0; i < QTILES; ++i) {
      mbar_init(&ctl->q_full[i], 1);
      mbar_init(&ctl->q_empty[i], 1);
    }
    for (int s = 0; s < KSTAGES; ++s) {
      mbar_init(&ctl->k_full[s], 1);
      mbar_init(&ctl->k_empty[s], 1);
    }
    for (int s = 0; s < VSTAGES; ++s) {
      mbar_init(&ctl->v_full[s], 1);
      mbar_init(&ctl->v_empty[s], 1);
    }
    fence_mbar_init();
    prefetch_tensormap(&tq);
    prefetch_tensormap(&tk);
    int w0 = 0, qb, bh;
    cta_unit(p, 0, w0);
    decode_unit(p, w0, qb, bh);
    for (int i = 0; i < QTILES; ++i) {
      mbar_arrive_expect_tx(&ctl->q_full[i], L::Q_BYTES);
#pragma unroll
      for (int d = 0; d < D / 64; ++d)
        tma_load_3d(smem + L::Q_OFF + i * L::Q_BYTES + d * (BM * 128), &tq, &ctl->q_full[i], d * 64,
                    qb * BQ + i * BM, bh);
      if (i == 0) {
        mbar_arrive_expect_tx(&ctl->k_full[0], L::KV_BYTES);
#pragma unroll
        for (int d = 0; d < D / 64; ++d)
          tma_load_3d(smem + L::K_OFF + d * (BN * 128), &tk, &ctl->k_full[0], d * 64, 0, bh);
      }
    }
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < QTILES; ++i) {
      mbar_init(&ctl->s_full[i], 1);
      mbar_init(&ctl->sm_done[i], SM_WARPS_PER_TILE);
      mbar_init(&ctl->p_lo[i], SM_WARPS_PER_TILE);
      mbar_init(&ctl->o_final[i], 1);
      mbar_init(&ctl->o_staged[i], SM_WARPS_PER_TILE);
    }
    mbar_init(&ctl->ostage_free, 1);
    mbar_init(&ctl->drain, 1);
    ctl->abort = 0;
    fence_mbar_init();
    prefetch_tensormap(&tv);
    prefetch_tensormap(&to);
  }
  if (warp == MMA_WARP) {
    tmem_alloc(&ctl->tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  if (warp >= 8) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(PER_REGS_OTHER) : "memory");
  if (warp == TMA_WARP) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      bool ok = true;
      // K and V run as one sequence each across units: sequence s uses stage s % 2.
      int k_issued = 1, v_issued = 0;  // the first unit's K_0 went out above
      int q_issued[QTILES] = {1, 1};  // loads into each Q buffer; the first unit's went out above
      auto load_k = [&](int row, int bh) -> bool {
        const int s = k_issued % KSTAGES;
        if (!mbar_wait_bounded(&ctl->k_empty[s], ((k_issued / KSTAGES) & 1) ^ 1, p.wait_limit, abort_flag))
          return false;
        mbar_arrive_expect_tx(&ctl->k_full[s], L::KV_BYTES);
#pragma unroll
        for (int d = 0; d < D / 64; ++d)
          tma_load_3d(smem + L::K_OFF + s * L::KV_BYTES + d * (BN * 128), &tk, &ctl->k_full[s], d * 64, row, bh);
        ++k_issued;
        return true;
      };
      auto load_v = [&](int row, int bh) -> bool {
        const int s = v_issued % VSTAGES;
        if (!mbar_wait_bounded(&ctl->v_empty[s], ((v_issued / VSTAGES) & 1) ^ 1, p.wait_limit, abort_flag))
          return false;
        mbar_arrive_expect_tx(&ctl->v_full[s], L::KV_BYTES);
#pragma unroll
        for (int d = 0; d < D / 64; ++d)
          tma_load_3d(smem + L::V_OFF + s * L::KV_BYTES + d * (BN * 128), &tv, &ctl->v_full[s], d * 64, row, bh);
        ++v_issued;
        return true;
      };
      // Q_i of unit u goes into Q_i's buffer once the last QK^T of tile i in unit u-1 retired.
      auto load_q = [&](int i, int u, int qb, int bh) -> bool {
        if (!mbar_wait_bounded(&ctl->q_empty[i], (u - 1) & 1, p.wait_limit, abort_flag)) return false;
        mbar_arrive_expect_tx(&ctl->q_full[i], L::Q_BYTES);
#pragma unroll
        for (int d = 0; d < D / 64; ++d)
          tma_load_3d(smem + L::Q_OFF + i * L::Q_BYTES + d * (BM * 128), &tq, &ctl->q_full[i], d * 64,
                      qb * BQ + i * BM, bh);
        ++q_issued[i];
        return true;
      };
      int w = 0;
      for (int u = 0; ok && cta_unit(p, u, w); ++u) {
        int qb, bh;
        decode_unit(p, w, qb, bh);
        const int n_max = max(kv_tiles(p, qb * BQ), kv_tiles(p, qb * BQ + BM));
        if (u > 0) {
          if (!load_q(0, u, qb, bh) || !load_k(0, bh) || !load_q(1, u, qb, bh)) {
            ok = false;
            break;
          }
        }
        int wn;
        if (cta_unit(p, u + 1, wn)) {  // the next unit's Q tiles into L2 while this unit runs
          int qb2, bh2;
          decode_unit(p, wn, qb2, bh2);
#pragma unroll
          for (int i = 0; i < QTILES; ++i)
            if (qb2 * BQ + i * BM < p.S)
#pragma unroll
              for (int d = 0; d < D / 64; ++d) tma_prefetch_3d(&tq, d * 64, qb2 * BQ + i * BM, bh2);
        }
        for (int j = 0; j < n_max && ok; ++j) {
          if (j + 1 < n_max && !load_k((j + 1) * BN, bh)) ok = false;
          else if (!load_v(j * BN, bh)) ok = false;
        }
      }
      if (!ok && !*abort_flag) fa2_abort(ctl, NTL_STATUS_TMA_EMPTY_WAIT);
      if (!ok) {
        // Drain every copy this thread issued before the CTA exits (the last load into each
        // buffer; earlier ones completed before their buffer was reused).
        for (int i = 0; i < QTILES; ++i)
          if (!mbar_wait_bounded(&ctl->q_full[i], (q_issued[i] - 1) & 1, int64_t(1) << 24, nullptr))
            atomicCAS(&g_fa2_status, 0u, NTL_STATUS_DRAIN_WAIT);
        for (int j = max(0, k_issued - KSTAGES); j < k_issued; ++j)
          if (!mbar_wait_bounded(&ctl->k_full[j % KSTAGES], (j / KSTAGES) & 1, int64_t(1) << 24, nullptr))
            atomicCAS(&g_fa2_status, 0u, NTL_STATUS_DRAIN_WAIT);
        for (int j = max(0, v_issued - VSTAGES); j < v_issued; ++j)
          if (!mbar_wait_bounded(&ctl->v_full[j % VSTAGES], (j / VSTAGES) & 1, int64_t(1) << 24, nullptr))
            atomicCAS(&g_fa2_status, 0u, NTL_STATUS_DRAIN_WAIT);
      }
    }
  } else if (warp == MMA_WARP) {
    // ------------------------------------------------------------------ MMA issuer
    if (elect_one_lane()) {
      constexpr uint32_t idesc_s = umma_idesc_f16_f32(BM, BN, 0, 0);  // B = K tile, K-major
      constexpr uint32_t idesc_o = umma_idesc_f16_f32(BM, D, 0, 1);   // B = V tile, N-major
      bool ok = true;
      // Unlike fa2_fwd_kernel's MMA thread, this one waits on the softmax hand-offs (p_lo,
      // sm_done) with try_wait, which may suspend it, rather than polling: its polls take issue
      // slots from the two softmax warps of its sub-partition, and this kernel's softmax steps
      // are the slower ones (+2.5% causal measured; the per-unit kernel measured 3% slower
      // suspending).
      auto wait_or_abort = [&](uint64_t* bar, uint32_t parity) -> bool {
        if (mbar_wait_bounded(bar, parity, p.wait_limit, abort_flag)) return true;
        if (!*abort_flag) fa2_abort(ctl, NTL_STATUS_MMA_FULL_WAIT);
        return false;
      };
      auto issue_s = [&](int i, int kseq) {  // S_i = Q_i K^T, K from ring sequence kseq
        const uint32_t q_addr = smem_u32(smem + L::Q_OFF + i * L::Q_BYTES);
        const uint32_t k_addr = smem_u32(smem + L::K_OFF + (kseq % KSTAGES) * L::KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
          tc_mma_f16_ss(tmem + L::S_COL(i), umma_desc_sw128(q_addr + off, 16, 1024),
                        umma_desc_sw128(k_addr + off, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
        }
        tc_commit(&ctl->s_full[i]);
      };
      int kbase = 0, vbase = 0;  // this unit's first K / V ring sequence
      int g[QTILES] = {0, 0};    // softmax steps of each tile before this unit
      int w = 0;
      for (int u = 0; ok && cta_unit(p, u, w); ++u) {
        int qb, bh;
        decode_unit(p, w, qb, bh);
        int n_t[QTILES];
#pragma unroll
        for (int i = 0; i < QTILES; ++i) n_t[i] = kv_tiles(p, qb * BQ + i * BM);
        const int n_max = max(n_t[0], n_t[1]);
        if (!wait_or_abort(&ctl->k_full[kbase % KSTAGES], (kbase / KSTAGES) & 1)) {
          ok = false;
          break;
        }
        for (int i = 0; i < QTILES && ok; ++i) {
          if (!wait_or_abort(&ctl->q_full[i], u & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (n_t[i] > 0) issue_s(i, kbase);
          if (n_t[i] <= 1) tc_commit(&ctl->q_empty[i]);  // Q_i is free once its last QK^T retires
        }
        if (!ok) break;
        tc_commit(&ctl->k_empty[kbase % KSTAGES]);  // K_0 is free once both QK^T retire
        for (int j = 0; j < n_max && ok; ++j) {
          const int vs = vbase + j, ks = kbase + j + 1;
          for (int i = 0; i < QTILES && ok; ++i) {
            if (j >= n_t[i]) continue;
            // V_j and K_{j+1} were loaded long before the softmax finishes: check them first,
            // so that only the softmax hand-off is on the critical path.
            if (!wait_or_abort(&ctl->v_full[vs % VSTAGES], (vs / VSTAGES) & 1)) {
              ok = false;
              break;
            }
            if (j + 1 < n_t[i] && !wait_or_abort(&ctl->k_full[ks % KSTAGES], (ks / KSTAGES) & 1)) {
              ok = false;
              break;
            }
            const uint32_t ph = static_cast<uint32_t>(g[i] + j) & 1u;
            if (!wait_or_abort(&ctl->p_lo[i], ph)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t v_addr = smem_u32(smem + L::V_OFF + (vs % VSTAGES) * L::KV_BYTES);
#pragma unroll
            for (int kk = 0; kk < BN / 32; ++kk)  // keys [0, 64): packed S columns [0, 32)
              tc_mma_f16_ts(tmem + L::O_COL(i), tmem + L::S_COL(i) + kk * 8,
                            umma_desc_sw128(v_addr + kk * 2048, BN * 128, 1024), idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
            if (!wait_or_abort(&ctl->sm_done[i], ph)) {
              ok = false;
              break;
            }
            tc_fence_after();
#pragma unroll
            for (int kk = BN / 32; kk < BN / 16; ++kk)  // keys [64, 128): packed S columns [32, 64)
              tc_mma_f16_ts(tmem + L::O_COL(i), tmem + L::S_COL(i) + kk * 8,
                            umma_desc_sw128(v_addr + kk * 2048, BN * 128, 1024), idesc_o, 1u);
            if (j == n_t[i] - 1) tc_commit(&ctl->o_final[i]);
            if (j + 1 < n_t[i]) {
              issue_s(i, ks);
              if (j + 2 == n_t[i]) tc_commit(&ctl->q_empty[i]);
            }
          }
          if (ok) {
            tc_commit(&ctl->v_empty[vs % VSTAGES]);                          // V_j consumed by both P V
            if (j + 1 < n_max) tc_commit(&ctl->k_empty[ks % KSTAGES]);       // K_{j+1} by both QK^T
          }
        }
        kbase += n_max;
        vbase += n_max;
#pragma unroll
        for (int i = 0; i < QTILES; ++i) g[i] += n_t[i];
      }
      if (!ok) {
        tc_commit(&ctl->drain);
        if (!mbar_wait_bounded(&ctl->drain, 0, int64_t(1) << 24, nullptr))
          atomicCAS(&g_fa2_status, 0u, NTL_STATUS_DRAIN_WAIT);
      }
    }
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(PER_REGS_SOFTMAX) : "memory");
    // ------------------------------------------------------------------ softmax warps
    // Warp w: query tile i = w/4; thread = row r = 32*(w%4) + lane = its TMEM lane (the lanes a
    // warp may access), all BN keys of the row in registers: row max and sum need no exchange.
    const int i = warp >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_addr = tmem + lane_off + L::S_COL(i);
    const uint32_t o_addr = tmem + lane_off + L::O_COL(i);
    const float c = p.c;
    const bool storer = quarter == 0 && lane == 0;
    uint8_t* ot = smem + L::OS_OFF;
    bool ok = true;
    int g = 0;  // this tile's softmax steps before the current unit
    int f = 0;  // units in which this tile had rows inside S
    int w = 0;
    for (int u = 0; ok && cta_unit(p, u, w); ++u) {
      int qb, bh;
      decode_unit(p, w, qb, bh);
      const int tile_q0 = qb * BQ + i * BM;
      const int qrow = tile_q0 + r;
      const int n_mine = kv_tiles(p, tile_q0);
      const int key_lim = p.causal ? min(p.S, qrow + 1) : p.S;  // keys < key_lim are kept
      float m_use = -INFINITY, l = 0.0f;
      for (int j = 0; j < n_mine; ++j) {
        const uint32_t ph = static_cast<uint32_t>(g + j) & 1u;
        if (!mbar_wait_bounded(&ctl->s_full[i], ph, p.wait_limit, abort_flag)) {
          if (!*abort_flag) fa2_abort(ctl, NTL_STATUS_SOFTMAX_WAIT);
          ok = false;
          break;
        }
        __syncwarp();
        tc_fence_after();
        uint32_t sv[BN];  // S[r, j*BN + k]
#pragma unroll
        for (int ch = 0; ch < BN / 32; ++ch)
          tmem_ld_32x32b_x32(s_addr + ch * 32, *reinterpret_cast<uint32_t(*)[32]>(sv + ch * 32));
        tc_wait_ld();
        if ((j * BN + BN > p.S) || (p.causal && j * BN + BN - 1 > tile_q0)) {
#pragma unroll
          for (int k = 0; k < BN; ++k)
            if (j * BN + k >= key_lim) sv[k] = __float_as_uint(-INFINITY);
        }
        float mx;
        {
          float x[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
          for (int k = 0; k < BN; k += 8) {
            x[0] = fmax3(x[0], __uint_as_float(sv[k]), __uint_as_float(sv[k + 1]));
            x[1] = fmax3(x[1], __uint_as_float(sv[k + 2]), __uint_as_float(sv[k + 3]));
            x[2] = fmax3(x[2], __uint_as_float(sv[k + 4]), __uint_as_float(sv[k + 5]));
            x[3] = fmax3(x[3], __uint_as_float(sv[k + 6]), __uint_as_float(sv[k + 7]));
          }
          mx = fmax3(fmaxf(x[0], x[1]), x[2], x[3]);
        }
        // lazy max
        float rs = 1.0f;
        bool moved = false;
        if (j == 0) {
          m_use = mx;
        } else if ((mx - m_use) * c > kRescaleLog2) {
          rs = ex2_approx((m_use - mx) * c);
          m_use = mx;
          moved = true;
        }
        if (__any_sync(0xffffffffu, moved)) {
          // O_i = P_{<j} V is complete: S_i of this tile was issued after the last P_i V.
#pragma unroll 1
          for (int ch = 0; ch < D / 32; ++ch) {
            uint32_t o[32];
            tmem_ld_32x32b_x32(o_addr + ch * 32, o);
            tc_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * rs);
            tmem_st_32x32b_x32(o_addr + ch * 32, o);
          }
        }
        // p = exp2(s*c - m*c) -> fp16 pairs: keys 2u, 2u+1 in S column u (columns already read)
        const uint64_t c2 = f2_make(c, c);
        const uint64_t nm2 = f2_make(-m_use * c, -m_use * c);
        uint64_t acc2[2] = {0ull, 0ull};
#pragma unroll
        for (int ch = 0; ch < BN / 32; ++ch) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int k = ch * 32 + 2 * e;
            const uint64_t x2 = f2_fma(f2_make(__uint_as_float(sv[k]), __uint_as_float(sv[k + 1])), c2, nm2);
            float p0, p1;
            if ((e & 3) == 3) {  // one pair in four on the FMA pipe
              exp2_fma2(x2, p0, p1);
            } else {
              float x0, x1;
              f2_split(x2, x0, x1);
              p0 = ex2_approx(x0);
              p1 = ex2_approx(x1);
            }
            acc2[e & 1] = f2_add(acc2[e & 1], f2_make(p0, p1));
            pk[e] = pack_half2(p0, p1);
          }
          tmem_st_32x32b_x16(s_addr + ch * 16, pk);
          if (ch == BN / 64 - 1) {
            // keys [0, BN/2) of P are in TMEM: the MMA warp may start on them
            tc_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ctl->p_lo[i]);
          }
        }
        float sum;
        {
          float u0, u1;
          f2_split(f2_add(acc2[0], acc2[1]), u0, u1);
          sum = u0 + u1;
        }
        l = (j == 0) ? sum : __fmaf_rn(l, rs, sum);
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->sm_done[i]);
      }
      if (!ok) break;
      // epilogue: O / l -> fp16.  Each thread writes its row into the staging buffer in the
      // layout of the 128-byte-swizzled tiles, and one thread stores the tile with one TMA
      // store per 64-column box (the tensor map clips rows past S).  The two tiles take the
      // buffer in turn (use 2u + i); a tile waits until the previous use has been read out.
      const int use = 2 * u + i;
      if (n_mine > 0) {
        if (!mbar_wait_bounded(&ctl->o_final[i], f & 1, p.wait_limit, abort_flag)) {
          if (!*abort_flag) fa2_abort(ctl, NTL_STATUS_SOFTMAX_WAIT);
          break;
        }
        __syncwarp();
        tc_fence_after();
        const float inv_l = 1.0f / l;
        uint32_t ov[D];  // the row of O: every chunk in flight before one wait
#pragma unroll
        for (int ch = 0; ch < D / 32; ++ch)
          tmem_ld_32x32b_x32(o_addr + ch * 32, *reinterpret_cast<uint32_t(*)[32]>(ov + ch * 32));
        tc_wait_ld();
        if (use > 0 && !mbar_wait_bounded(&ctl->ostage_free, (use - 1) & 1, p.wait_limit, abort_flag)) {
          if (!*abort_flag) fa2_abort(ctl, NTL_STATUS_SOFTMAX_WAIT);
          break;
        }
#pragma unroll
        for (int ch = 0; ch < D / 32; ++ch) {
          uint32_t hv[16];
#pragma unroll
          for (int e = 0; e < 16; ++e)
            hv[e] = pack_half2(__uint_as_float(ov[ch * 32 + 2 * e]) * inv_l,
                               __uint_as_float(ov[ch * 32 + 2 * e + 1]) * inv_l);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const int u16 = ch * 4 + q4;  // 16-byte unit of the row; 8 units per 64-column box
            uint8_t* dst = ot + (u16 >> 3) * (BM * 128) + r * 128 + (((u16 & 7) ^ (r & 7)) << 4);
            *reinterpret_cast<uint4*>(dst) = make_uint4(hv[4 * q4], hv[4 * q4 + 1], hv[4 * q4 + 2], hv[4 * q4 + 3]);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->o_staged[i]);
        if (storer) {
          if (mbar_wait_bounded(&ctl->o_staged[i], f & 1, p.wait_limit, abort_flag)) {
#pragma unroll
            for (int d = 0; d < D / 64; ++d) tma_store_3d(&to, ot + d * (BM * 128), d * 64, tile_q0, bh);
            bulk_commit();
            bulk_wait_read();
            mbar_arrive(&ctl->ostage_free);
          } else {
            if (!*abort_flag) fa2_abort(ctl, NTL_STATUS_SOFTMAX_WAIT);
            break;
          }
        }
        ++f;
      } else if (storer) {
        // No rows of this tile inside S: pass the buffer on without a store.
        if (use > 0 && !mbar_wait_bounded(&ctl->ostage_free, (use - 1) & 1, p.wait_limit, abort_flag)) {
          if (!*abort_flag) fa2_abort(ctl, NTL_STATUS_SOFTMAX_WAIT);
          break;
        }
        mbar_arrive(&ctl->ostage_free);
      }
      g += n_mine;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == MMA_WARP) tmem_dealloc(tmem, TMEM_COLS);
}

// ------------------------------------------------------------------------- host side

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// [B*H, S, D] fp16, box {64, 128, 1}, 128-byte swizzle.
int make_map_bshd(CUtensorMap* map, const void* base, uint64_t bh, uint64_t s, uint64_t d) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return ntl_fail(NTL_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[3] = {d, s, bh};
  cuuint64_t strides[2] = {d * 2, s * d * 2};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return ntl_fail(NTL_ERR_CUDA, "cuTensorMapEncodeTiled (attention) failed (%d)", int(r));
  return NTL_OK;
}

int set_smem_once(const void* kernel, int bytes, std::atomic<uint64_t>& done_mask) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return ntl_fail(NTL_ERR_CUDA, "cudaGetDevice failed");
  const uint64_t bit = dev < 64 ? (uint64_t(1) << dev) : 0;
  if (!(bit && (done_mask.load(std::memory_order_acquire) & bit))) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return ntl_fail(NTL_ERR_CUDA, "cudaFuncSetAttribute(fa2): %s", cudaGetErrorString(e));
    done_mask.fetch_or(bit, std::memory_order_release);
  }
  // The in-kernel register split (8 softmax warps up, 4 warps down) must equal what the launch
  // allocates (384 threads x REGS_LAUNCH), or the raising warps would wait for registers
  // forever: refuse to launch a build whose register count differs.
  cudaFuncAttributes fa;
  if (cudaFuncGetAttributes(&fa, kernel) != cudaSuccess || fa.numRegs != REGS_LAUNCH)
    return ntl_fail(NTL_ERR_UNSUPPORTED, "attention: kernel compiled with %d registers, the split needs %d",
                    fa.numRegs, REGS_LAUNCH);
  return NTL_OK;
}

template <int D>
int launch_fa2(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mo,
               const Fa2Params& p, cudaStream_t s) {
  static std::atomic<uint64_t> done_mask{0};
  if (int rc = set_smem_once(reinterpret_cast<const void*>(fa2_fwd_kernel<D>), Fa2Smem<D>::BYTES, done_mask)) return rc;
  const unsigned grid = static_cast<unsigned>(p.n_qb) * static_cast<unsigned>(p.BH);
  fa2_fwd_kernel<D><<<grid, THREADS, Fa2Smem<D>::BYTES, s>>>(mq, mk, mv, mo, p);
  ntl_note_launch();
  return ntl_check_launch("attention launch");
}

template <int D>
int launch_fa2_persist(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mo,
                       const PersistParams& p, int sms, cudaStream_t s) {
  static std::atomic<uint64_t> done_mask{0};
  if (int rc = set_smem_once(reinterpret_cast<const void*>(fa2_persist_kernel<D>), PersistSmem<D>::BYTES, done_mask))
    return rc;
  // One CTA per SM, and no more CTAs than pairs of units, so that every CTA's first unit
  // (2 * blockIdx.x) exists: its loads are issued before the CTA-wide sync.
  const int pairs = (p.units + 1) / 2;
  const unsigned grid = static_cast<unsigned>(pairs < sms ? pairs : sms);
  fa2_persist_kernel<D><<<grid, THREADS, PersistSmem<D>::BYTES, s>>>(mq, mk, mv, mo, p);
  ntl_note_launch();
  return ntl_check_launch("attention launch");
}

}  // namespace

static std::atomic<int> g_causal_grid{NTL_FA2_GRID_AUTO};  // ntl_fa2_set_causal_grid

extern "C" int ntl_fa2_set_causal_grid(int mode) {
  NTL_REQUIRE(mode == NTL_FA2_GRID_AUTO || mode == NTL_FA2_GRID_PERSISTENT || mode == NTL_FA2_GRID_PER_BLOCK,
              NTL_ERR_INVALID, "attention: causal grid mode %d is not one of 0 (auto), 1 (persistent), 2 (per block)",
              mode);
  g_causal_grid.store(mode, std::memory_order_relaxed);
  return NTL_OK;
}

uint32_t ntl_fa2_status_read(int clear) {
  uint32_t v = 0;
  if (cudaMemcpyFromSymbol(&v, g_fa2_status, sizeof(v)) != cudaSuccess) return 0;
  if (clear) {
    uint32_t z = 0;
    cudaMemcpyToSymbol(g_fa2_status, &z, sizeof(z));
  }
  return v;
}

extern "C" int ntl_fa2_fwd_f16(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* o, int64_t batch,
                               int64_t heads, int64_t seq, int64_t dim, float scale_log2, int causal,
                               ntl_stream_t stream) {
  NTL_REQUIRE(batch >= 0 && heads >= 0 && seq >= 0 && dim >= 0, NTL_ERR_INVALID, "attention: negative size");
  NTL_REQUIRE(dim == 64 || dim == 128, NTL_ERR_UNSUPPORTED, "attention: head_dim %lld is not supported (64 or 128)",
              (long long)dim);
  if (batch == 0 || heads == 0 || seq == 0) return NTL_OK;
  NTL_REQUIRE(q && k && v && o, NTL_ERR_INVALID, "attention: NULL pointer");
  NTL_REQUIRE(ntl_aligned(q, 16) && ntl_aligned(k, 16) && ntl_aligned(v, 16) && ntl_aligned(o, 16), NTL_ERR_ALIGNMENT,
              "attention: Q, K, V, O must be 16-byte aligned");
  NTL_REQUIRE(seq < (int64_t(1) << 31), NTL_ERR_UNSUPPORTED, "attention: sequence too long");
  NTL_REQUIRE(((seq + BQ - 1) / BQ) * batch * heads < (int64_t(1) << 31), NTL_ERR_UNSUPPORTED,
              "attention: more than 2^31 - 1 (batch, head, 256-query block) blocks");
  CUtensorMap mq, mk, mv, mo;
  const uint64_t bh = static_cast<uint64_t>(batch * heads);
  if (int rc = make_map_bshd(&mq, q, bh, seq, dim)) return rc;
  if (int rc = make_map_bshd(&mk, k, bh, seq, dim)) return rc;
  if (int rc = make_map_bshd(&mv, v, bh, seq, dim)) return rc;
  if (int rc = make_map_bshd(&mo, o, bh, seq, dim)) return rc;
  int sms = 0;
  if (int rc = ntl_num_sms(&sms)) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Causal runs on the persistent grid when its equal-cost pairs of units fill the SMs' rounds:
  // pairs / (rounds x SMs) >= kPersistMinFill.  Below that (the 512 or 256 pairs of a [2 or 1,
  // 32, 4096] shard leave the last of 4 or 2 rounds 46% full) the one-CTA-per-unit grid, which
  // the hardware balances block by block, measured 5.4% faster; at [8, 32, 4096] (2048 pairs,
  // 0.99 full) the persistent grid is 2-4% faster.
  const int64_t units = ((seq + BQ - 1) / BQ) * batch * heads;
  const int64_t pairs = (units + 1) / 2;
  const int64_t rounds = (pairs + sms - 1) / sms;
  const int grid_mode = g_causal_grid.load(std::memory_order_relaxed);
  const bool persistent = causal && (grid_mode == NTL_FA2_GRID_PERSISTENT ||
                                     (grid_mode == NTL_FA2_GRID_AUTO &&
                                      pairs >= kPersistMinFill * static_cast<double>(rounds * sms)));
  if (persistent) {
    PersistParams pp;
    pp.S = static_cast<int>(seq);
    pp.n_qb = static_cast<int>((seq + BQ - 1) / BQ);
    pp.BH = static_cast<int>(batch * heads);
    pp.units = pp.n_qb * pp.BH;
    pp.causal = 1;
    pp.c = scale_log2;
    pp.wait_limit = ntl_wait_limit();
    if (dim == 64) return launch_fa2_persist<64>(mq, mk, mv, mo, pp, sms, s);
    return launch_fa2_persist<128>(mq, mk, mv, mo, pp, sms, s);
  }
  Fa2Params p;
  p.o = reinterpret_cast<__half*>(o);
  p.S = static_cast<int>(seq);
  p.n_qb = static_cast<int>((seq + BQ - 1) / BQ);
  p.BH = static_cast<int>(batch * heads);
  p.causal = causal ? 1 : 0;
  p.c = scale_log2;
  p.succ_stride = sms;  // one CTA per SM
  p.wait_limit = ntl_wait_limit();
  if (dim == 64) return launch_fa2<64>(mq, mk, mv, mo, p, s);
  return launch_fa2<128>(mq, mk, mv, mo, p, s);
}
