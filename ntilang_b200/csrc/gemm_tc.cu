// FP16 GEMM with fp32 accumulation and a fused epilogue, sm_100a.
//
// Reference: the GEMM its emitter builds for examples/matmul.py:17-29 (codegen.py:969-1026
// mma.sync m16n8k16 + ldmatrix, :1611-1693 cp.async pipeline, :1280-1316 raster swizzle)
// and the fused epilogue of examples/matmul_relu.py:31-38 (codegen.py:1694-1734).
//
// Design (one CTA per SM, persistent):
//   warp 0      TMA producer: A tile 128x64 (K-major) and B tile 64x256 (N-major, or K-major
//               for transpose_B) into a 4-stage ring of 128B-swizzled smem stages.
//   warp 1      allocates 512 TMEM columns (two 128x256 fp32 accumulators), one elected
//               lane issues tcgen05.mma (M=128, N=256, K=16) and tcgen05.commit's the stage
//               back to the producer / the accumulator to the epilogue.
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns, alpha / bias / ReLU in registers,
//               128-bit stores to C.  The double-buffered accumulator lets the epilogue of
//               tile i overlap the main loop of tile i+1.
// Work schedule: whole waves of output tiles are data-parallel (one CTA computes a tile over
// all of K).  With a workspace (ntl_gemm_f16_f32_ws), the tiles of the last, partial wave
// are split along K: here (M <= 128) evenly over all CTAs (stream-K), in the CTA-pair kernel
// below (M > 128) into 2-4 equal pieces on otherwise idle pairs.  A CTA whose range starts
// mid-K writes its fp32 partial sum to a workspace slot and raises a flag; the CTA holding the
// tile's first k-block waits for those flags (bounded), adds the partials and runs the
// epilogue.  Without a workspace every tile is data-parallel.
// Every mbarrier / flag wait is bounded (ntl_set_wait_limit and a 2 s wall-clock cap); a
// wait that gives up records a status code, raises the CTA abort flag, drains in-flight TMA
// loads and MMAs, frees TMEM and returns.  Shapes TMA cannot address (K or N not a
// multiple of 8, unaligned pointers) use a CUDA-core tiled kernel with the same epilogue.
#include <algorithm>
#include <atomic>
#include <mutex>

#include "ntl_common.cuh"

namespace {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_STAGE = BM * BK * 2;        // 16 KB
constexpr int B_STAGE = BN * BK * 2;        // 32 KB
constexpr int STAGE_BYTES = A_STAGE + B_STAGE;
constexpr int THREADS = 192;
constexpr int TMEM_COLS = 512;
// Per epilogue warp, the bias values of the current tile's BN columns (bias[N] form).
constexpr int BIAS_SMEM_BYTES = 4 * BN * 4;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*barriers*/ + BIAS_SMEM_BYTES + 1024 /*alignment slack*/;
constexpr int GROUP_M = 8;
constexpr int SK_MIN_UNITS = 8;             // fewest k-blocks a stream-K CTA takes
constexpr size_t SK_SLOT_FLOATS = size_t(BM) * BN;
// Workspace layout shared by every plan: a fixed block of flag words first (so that the
// flags of one shape never land on another shape's partial sums when a workspace is reused),
// then the partial-sum slots of SK_SLOT_FLOATS floats each.
constexpr size_t kWsFlagBytes = 4096;
constexpr size_t kWsMaxSlots = kWsFlagBytes / 4;

__device__ uint32_t g_gemm_status;

struct GemmParams {
  float* c;
  const float* bias;
  int bias_mode;
  float alpha;
  int relu;
  int M, N, K;
  int b_trans;
  int vec_store;  // C rows 16-byte aligned
  int vec_bias;   // bias 16-byte aligned and N % 4 == 0
  int64_t wait_limit;
  // work plan
  int num_m, num_n, kb;  // tile grid and k-blocks per tile
  int dp_tiles;          // tiles [0, dp_tiles) are data-parallel
  int sk_ctas;           // CTAs [0, sk_ctas) share the k-blocks of tiles [dp_tiles, tiles)
  int64_t sk_units;
  float* ws;             // sk_ctas partial-sum slots of BM x BN fp32
  uint32_t* flags;       // sk_ctas flags (0 = empty, 1 = partial ready)
  int nar_pairs;         // CTA-pair kernel: pairs [0, nar_pairs) each take one column half of a tail tile
};

struct __align__(8) SharedCtl {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint64_t sk_stored;  // epilogue warps finished writing a partial
  uint64_t sk_read;    // epilogue warps saw every contributor flag of a finalised tile
  uint32_t tmem_base;
  int abort;
};

struct Work {
  int tile;
  int k0, k1;  // k-block range [k0, k1)
};

// The ordered list of work items of one CTA: its data-parallel tiles, then its stream-K
// segments.  Every role walks the same list.
struct WorkIter {
  int t;
  int64_t u, u_end;
  __device__ __forceinline__ static int64_t sk_begin(const GemmParams& p, int cta) {
    return cta >= p.sk_ctas ? p.sk_units : (p.sk_units * cta) / p.sk_ctas;
  }
  __device__ __forceinline__ void init(const GemmParams& p) {
    t = blockIdx.x;
    u = sk_begin(p, blockIdx.x);
    u_end = sk_begin(p, blockIdx.x + 1);
    if (static_cast<int>(blockIdx.x) >= p.sk_ctas) u = u_end = 0;
  }
  __device__ __forceinline__ bool next(const GemmParams& p, Work& w) {
    if (t < p.dp_tiles) {
      w.tile = t, w.k0 = 0, w.k1 = p.kb;
      t += gridDim.x;
      return true;
    }
    if (u < u_end) {
      const int64_t local = u / p.kb;
      w.tile = p.dp_tiles + static_cast<int>(local);
      w.k0 = static_cast<int>(u - local * p.kb);
      const int64_t rest = u_end - u;
      w.k1 = rest < static_cast<int64_t>(p.kb - w.k0) ? w.k0 + static_cast<int>(rest) : p.kb;
      u += w.k1 - w.k0;
      return true;
    }
    return false;
  }
};

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& mb, int& nb) {
  const int per_group = GROUP_M * num_n;
  const int g = t / per_group;
  const int first = g * GROUP_M;
  const int size = min(num_m - first, GROUP_M);
  const int r = t % per_group;
  mb = first + r % size;
  nb = r / size;
}

__device__ __forceinline__ void record_abort(SharedCtl* ctl, uint32_t code) {
  atomicCAS(&g_gemm_status, 0u, code);
  *reinterpret_cast<volatile int*>(&ctl->abort) = 1;
}

// v = acc * alpha + b as two rounded ops (the program's order), then optional ReLU.
__device__ __forceinline__ float epi(float acc, float alpha, float b, int relu, int has_bias) {
  float v = alpha == 1.0f ? acc : __fmul_rn(acc, alpha);
  if (has_bias) v = __fadd_rn(v, b);
  return relu ? fmaxf(v, 0.0f) : v;
}

// bias[n0 .. n0 + BN) (zero past N) -> this warp's shared-memory copy, read back by broadcast
// in store_row_chunk.  One pass of 128-bit loads per tile instead of one load per output.
__device__ __forceinline__ void stage_bias_n(const GemmParams& p, int n0, float* bias_s, int lane) {
#pragma unroll
  for (int c = lane * 4; c < BN; c += 128) {
    const int col = n0 + c;
    float4 t;
    if (p.vec_bias && col + 3 < p.N) {
      t = __ldg(reinterpret_cast<const float4*>(p.bias + col));
    } else {
      t.x = col < p.N ? __ldg(p.bias + col) : 0.0f;
      t.y = col + 1 < p.N ? __ldg(p.bias + col + 1) : 0.0f;
      t.z = col + 2 < p.N ? __ldg(p.bias + col + 2) : 0.0f;
      t.w = col + 3 < p.N ? __ldg(p.bias + col + 3) : 0.0f;
    }
    *reinterpret_cast<float4*>(bias_s + c) = t;
  }
  __syncwarp();
}

// Epilogue of 32 accumulator columns [col0, col0+32) of one output row: alpha, bias, ReLU,
// then 128-bit stores when the row is 16-byte aligned and the chunk lies inside C.
// bias_chunk: the chunk's 32 bias[N] values in shared memory (bias[N] form only).
__device__ __forceinline__ void store_row_chunk(float (&v)[32], const GemmParams& p, int row, int col0, float* crow,
                                                float row_bias, const float* bias_chunk) {
  if (p.bias_mode == NTL_BIAS_MN && p.vec_bias && col0 + 32 <= p.N) {
    const float4* brow = reinterpret_cast<const float4*>(p.bias + static_cast<int64_t>(row) * p.N + col0);
    float4 b4[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) b4[q] = __ldg(brow + q);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      v[4 * q] = epi(v[4 * q], p.alpha, b4[q].x, p.relu, 1);
      v[4 * q + 1] = epi(v[4 * q + 1], p.alpha, b4[q].y, p.relu, 1);
      v[4 * q + 2] = epi(v[4 * q + 2], p.alpha, b4[q].z, p.relu, 1);
      v[4 * q + 3] = epi(v[4 * q + 3], p.alpha, b4[q].w, p.relu, 1);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      float b = row_bias;
      const int col = col0 + j;
      if (p.bias_mode == NTL_BIAS_N) b = bias_chunk[j];
      else if (p.bias_mode == NTL_BIAS_MN) b = (col < p.N) ? __ldg(p.bias + static_cast<int64_t>(row) * p.N + col) : 0.0f;
      v[j] = epi(v[j], p.alpha, b, p.relu, p.bias_mode);
    }
  }
  if (p.vec_store && col0 + 32 <= p.N) {
#pragma unroll
    for (int j = 0; j < 32; j += 4)
      *reinterpret_cast<float4*>(crow + col0 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (col0 + j < p.N) crow[col0 + j] = v[j];
  }
}

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait for a stream-K contributor flag (2 s wall-clock cap, abort-aware).
__device__ __forceinline__ bool wait_flag(const uint32_t* flag, int64_t limit, volatile int* abort_flag) {
  const uint64_t t0 = global_ns();
  for (int64_t i = 0; i < limit; ++i) {
    if (ld_acquire_u32(flag) != 0u) return true;
    if ((i & 63) == 63) {
      if (*abort_flag) return false;
      if (global_ns() - t0 > kWaitCapNs) return false;
      __nanosleep(64);
    }
  }
  return false;
}

__global__ void __launch_bounds__(THREADS, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_a,
                                                             const __grid_constant__ CUtensorMap tmap_b,
                                                             const GemmParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_STAGE;
  SharedCtl* ctl = reinterpret_cast<SharedCtl*>(smem + STAGES * STAGE_BYTES);
  volatile int* abort_flag = &ctl->abort;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&ctl->acc_full[a], 1);
      mbar_init(&ctl->acc_empty[a], 4);  // one arrival per epilogue warp
    }
    mbar_init(&ctl->drain, 1);
    mbar_init(&ctl->sk_stored, 4);
    mbar_init(&ctl->sk_read, 4);
    ctl->abort = 0;
    fence_mbar_init();
    prefetch_tensormap(&tmap_a);
    prefetch_tensormap(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(&ctl->tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = ctl->tmem_base;
  // Launched with programmatic stream serialization (no workspace): the setup above overlaps
  // the previous kernel on the stream; every global access (A, B, bias, C) comes after this.
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one_lane()) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      WorkIter it;
      it.init(p);
      Work w;
      while (ok && it.next(p, w)) {
        int mb, nb;
        tile_coords(w.tile, p.num_m, p.num_n, mb, nb);
        const int m0 = mb * BM, n0 = nb * BN;
        for (int kb = w.k0; kb < w.k1; ++kb) {
          if (!mbar_wait_bounded(&ctl->empty[stage], phase ^ 1, p.wait_limit, abort_flag)) {
            if (!*abort_flag) record_abort(ctl, NTL_STATUS_TMA_EMPTY_WAIT);
            ok = false;
            break;
          }
          uint8_t* a_dst = sA + stage * A_STAGE;
          uint8_t* b_dst = sB + stage * B_STAGE;
          mbar_arrive_expect_tx(&ctl->full[stage], STAGE_BYTES);
          tma_load_2d(a_dst, &tmap_a, &ctl->full[stage], kb * BK, m0);
          if (p.b_trans) {
            tma_load_2d(b_dst, &tmap_b, &ctl->full[stage], kb * BK, n0);
          } else {
#pragma unroll
            for (int i = 0; i < BN / 64; ++i)
              tma_load_2d(b_dst + i * (64 * BK * 2), &tmap_b, &ctl->full[stage], n0 + i * 64, kb * BK);
          }
          ++issued;
          if (++stage == STAGES) stage = 0, phase ^= 1;
        }
      }
      if (!ok) {
        // Drain: the last min(issued, STAGES) stages may still have loads in flight.
        int s = stage;
        uint32_t ph = phase;
        for (int i = 0; i < STAGES && i < issued; ++i) {
          if (--s < 0) s = STAGES - 1, ph ^= 1;
          if (!mbar_wait_bounded(&ctl->full[s], ph, int64_t(1) << 24, nullptr))
            atomicCAS(&g_gemm_status, 0u, NTL_STATUS_DRAIN_WAIT);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one_lane()) {
      const uint32_t idesc = umma_idesc_f16_f32(BM, BN, 0, p.b_trans ? 0 : 1);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      WorkIter it;
      it.init(p);
      Work w;
      for (; ok && it.next(p, w); ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait_bounded(&ctl->acc_empty[acc], acc_phase ^ 1, p.wait_limit, abort_flag)) {
          if (!*abort_flag) record_abort(ctl, NTL_STATUS_ACC_EMPTY_WAIT);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = w.k0; kb < w.k1; ++kb) {
          if (!mbar_wait_bounded(&ctl->full[stage], phase, p.wait_limit, abort_flag)) {
            if (!*abort_flag) record_abort(ctl, NTL_STATUS_MMA_FULL_WAIT);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * A_STAGE);
          const uint32_t b_addr = smem_u32(sB + stage * B_STAGE);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t adesc = umma_desc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t bdesc = p.b_trans ? umma_desc_sw128(b_addr + k * 32, 16, 1024)
                                             : umma_desc_sw128(b_addr + k * 2048, 64 * BK * 2, 1024);
            tc_mma_f16_ss(d_tmem, adesc, bdesc, idesc, (kb > w.k0 || k > 0) ? 1u : 0u);
          }
          tc_commit(&ctl->empty[stage]);
          if (++stage == STAGES) stage = 0, phase ^= 1;
        }
        if (!ok) break;
        tc_commit(&ctl->acc_full[acc]);
      }
      // Drain: every MMA this thread issued retires before TMEM is freed, also when another
      // role gave up after the last issue.
      tc_commit(&ctl->drain);
      if (!mbar_wait_bounded(&ctl->drain, 0, int64_t(1) << 24, nullptr))
        atomicCAS(&g_gemm_status, 0u, NTL_STATUS_DRAIN_WAIT);
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..5)
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31 are accessible to this warp
    const int r_local = quarter * 32 + lane;
    int local = 0;
    int finalised = 0;  // stream-K tiles finalised so far (phase of sk_read)
    WorkIter it;
    it.init(p);
    Work w;
    for (; it.next(p, w); ++local) {
      int mb, nb;
      tile_coords(w.tile, p.num_m, p.num_n, mb, nb);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait_bounded(&ctl->acc_full[acc], acc_phase, p.wait_limit, abort_flag)) {
        if (!*abort_flag) record_abort(ctl, NTL_STATUS_ACC_FULL_WAIT);
        break;
      }
      __syncwarp();
      tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
      if (w.k0 > 0) {
        // Stream-K contributor: raw partial sums -> this CTA's workspace slot, then its flag.
        // Slot layout [column quad][row][4]: a warp's float4 stores are 512 contiguous bytes.
        float4* slot = reinterpret_cast<float4*>(p.ws + static_cast<size_t>(blockIdx.x) * SK_SLOT_FLOATS) + r_local;
        for (int chunk = 0; chunk < BN / 32; ++chunk) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + chunk * 32, r);
          tc_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            __stcg(slot + static_cast<size_t>(chunk * 8 + j / 4) * BM,
                   make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]),
                               __uint_as_float(r[j + 3])));
        }
        __threadfence();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->acc_empty[acc]);
        if (lane == 0) mbar_arrive(&ctl->sk_stored);
        if (warp == 2 && lane == 0) {
          if (mbar_wait_bounded(&ctl->sk_stored, 0, p.wait_limit, abort_flag)) {
            __threadfence();
            atomicExch(p.flags + blockIdx.x, 1u);
          } else if (!*abort_flag) {
            record_abort(ctl, NTL_STATUS_ACC_FULL_WAIT);
          }
        }
        continue;
      }
      // Contributors of this tile (stream-K finaliser): CTAs after this one whose range starts
      // inside the tile.
      int first_c = 0, last_c = -1;
      if (w.k1 < p.kb) {
        const int64_t tile_end_u = static_cast<int64_t>(w.tile - p.dp_tiles + 1) * p.kb;
        first_c = blockIdx.x + 1;
        last_c = blockIdx.x;
        while (last_c + 1 < p.sk_ctas && WorkIter::sk_begin(p, last_c + 1) < tile_end_u) ++last_c;
        bool ready = true;
        for (int cc = first_c; cc <= last_c && ready; ++cc) {
          if (lane == 0) ready = wait_flag(p.flags + cc, p.wait_limit, abort_flag);
          ready = __shfl_sync(0xffffffffu, ready ? 1 : 0, 0) != 0;
        }
        if (!ready) {
          if (!*abort_flag) record_abort(ctl, NTL_STATUS_ACC_FULL_WAIT);
          break;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->sk_read);
      }
      const int row = mb * BM + r_local;
      const bool row_ok = row < p.M;
      float* crow = p.c + static_cast<int64_t>(row) * p.N;
      const float row_bias = (p.bias_mode == NTL_BIAS_M && row_ok) ? __ldg(p.bias + row) : 0.0f;
      float* bias_s = reinterpret_cast<float*>(smem + STAGES * STAGE_BYTES + 1024) + (warp - 2) * BN;
      if (p.bias_mode == NTL_BIAS_N) stage_bias_n(p, nb * BN, bias_s, lane);
      for (int chunk = 0; chunk < BN / 32; ++chunk) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + chunk * 32, r);
        tc_wait_ld();
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        for (int cc = first_c; cc <= last_c; ++cc) {
          const float4* part = reinterpret_cast<const float4*>(p.ws + static_cast<size_t>(cc) * SK_SLOT_FLOATS) + r_local;
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            const float4 q = __ldcg(part + static_cast<size_t>(chunk * 8 + j / 4) * BM);
            v[j] += q.x, v[j + 1] += q.y, v[j + 2] += q.z, v[j + 3] += q.w;
          }
        }
        const int col0 = nb * BN + chunk * 32;
        if (!row_ok || col0 >= p.N) continue;
        store_row_chunk(v, p, row, col0, crow, row_bias, bias_s + chunk * 32);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->acc_empty[acc]);
      if (last_c >= first_c) {
        // Every epilogue warp has seen the flags: reset them for the next launch.
        if (warp == 2 && lane == 0) {
          if (mbar_wait_bounded(&ctl->sk_read, finalised & 1, p.wait_limit, abort_flag)) {
            for (int cc = first_c; cc <= last_c; ++cc) atomicExch(p.flags + cc, 0u);
          } else if (!*abort_flag) {
            record_abort(ctl, NTL_STATUS_ACC_FULL_WAIT);
          }
        }
        ++finalised;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, TMEM_COLS);
}

// ------------------------------------------------------------------ CTA-pair kernel
// The same GEMM on clusters of two CTAs (two SMs) that share one tcgen05 MMA of
// M=256 x N=256 x K=16 (cta_group::2).  The even CTA (rank 0) issues the MMAs; each CTA
// holds 128 rows of the pair's A tile and 128 columns of its B tile in its own shared
// memory, and 128 rows x 256 columns of the accumulator in its own TMEM.  Per k-block an SM
// loads 32 KB instead of the 48 KB of the one-SM kernel for the same tensor work, which is
// what bounds that kernel (its loads from L2 run at the SM's operand bandwidth).
//   warp 0 (both CTAs)  TMA: own A rows and own B columns; completion is counted on the
//                       even CTA's `full` barrier, which that CTA arms for both halves.
//   warp 1 (rank 0)     MMA issue; commits release `empty` and signal `acc_full` in both
//                       CTAs (commit multicast, no multicast loads).
//   warps 2..5          epilogue of the CTA's 128 rows; they free an accumulator by
//                       arriving on the even CTA's `acc_empty` (8 arrivals).
// With a workspace, the last partial wave's tiles are split along K (PairIter); a split
// tile's piece 0 adds the other pieces' partial sums (workspace slots behind bounded flag
// waits) before its epilogue.
// Teardown: both CTAs meet at a cluster barrier; if any role gave up, the even CTA's
// producer balances and waits out every stage load either CTA still has in flight (it knows
// both issue counts), then both meet again before TMEM is freed.
constexpr int PR_TILE_M = 256;                   // rows of a pair tile (128 per CTA)
constexpr int PR_BM = 128;
constexpr int PR_BN_HALF = BN / 2;               // B columns held by one CTA
constexpr int PR_STAGES = 6;
constexpr int PR_A_STAGE = PR_BM * BK * 2;       // 16 KB
constexpr int PR_B_STAGE = PR_BN_HALF * BK * 2;  // 16 KB
constexpr int PR_STAGE_BYTES = PR_A_STAGE + PR_B_STAGE;
constexpr int PR_SMEM_BYTES = PR_STAGES * PR_STAGE_BYTES + 1024 + BIAS_SMEM_BYTES + 1024;
static_assert(PR_SMEM_BYTES <= 227 * 1024, "pair kernel shared memory");

struct __align__(8) PairCtl {
  uint64_t full[PR_STAGES];   // rank 0: both CTAs' loads of a stage landed
  uint64_t empty[PR_STAGES];  // each CTA: the MMAs reading the stage retired
  uint64_t acc_full[2];       // each CTA: accumulator complete
  uint64_t acc_empty[2];      // rank 0: the 8 epilogue warps of the pair drained it
  uint64_t drain;
  uint64_t sk_stored;         // each CTA: its 4 epilogue warps wrote a partial sum
  uint64_t sk_read;           // each CTA: its 4 epilogue warps read every contributor flag
  uint32_t tmem_base;
  int abort;
  int issued;       // rank 0: stage loads its producer issued
  int peer_issued;  // rank 0: stage loads the odd CTA's producer issued
};

// Work of one pair: its data-parallel tiles (tile = pair + i * pairs < dp_tiles), then at most
// one K-piece of a split tile.  The last partial wave's tiles (dp_tiles .. tiles) are each split
// into `split` = p.sk_units K-ranges over p.sk_ctas = (tiles - dp_tiles) * split pairs; in each
// group of `split` consecutive pairs the highest one holds piece 0 (k-blocks from 0) and
// finalises the tile, so every pair it waits for was launched before it.
// Without a workspace the last partial wave's tiles are instead split along N: pair q of
// [0, nar_pairs) computes columns [128 h, 128 h + 128) of tail tile dp_tiles + q / 2 (h = q % 2)
// as a 256 x 128 MMA, so the tail takes half a tile's time and needs no partial sums.
struct PairWork {
  int tile, k0, k1;
  int piece;  // 0: data-parallel or finaliser; > 0: contributor
  int slot;   // first workspace slot of this tile's contributors (split tiles only)
  int half;   // -1: all BN columns; 0 / 1: that 128-column half (N-split tail tile)
};

struct PairIter {
  int t;
  bool split_left, narrow_left;
  __device__ __forceinline__ void init(const GemmParams& p, int pair) {
    t = pair;
    split_left = pair < p.sk_ctas;
    narrow_left = pair < p.nar_pairs;
  }
  __device__ __forceinline__ bool next(const GemmParams& p, int pair, int num_pairs, PairWork& w) {
    w.half = -1;
    if (t < p.dp_tiles) {
      w.tile = t, w.k0 = 0, w.k1 = p.kb, w.piece = 0, w.slot = 0;
      t += num_pairs;
      return true;
    }
    if (narrow_left) {
      narrow_left = false;
      w.tile = p.dp_tiles + pair / 2, w.half = pair % 2;
      w.k0 = 0, w.k1 = p.kb, w.piece = 0, w.slot = 0;
      return true;
    }
    if (split_left) {
      split_left = false;
      const int split = static_cast<int>(p.sk_units);
      const int tl = pair / split;
      w.piece = (split - 1) - pair % split;
      w.tile = p.dp_tiles + tl;
      w.k0 = static_cast<int>(static_cast<int64_t>(p.kb) * w.piece / split);
      w.k1 = static_cast<int>(static_cast<int64_t>(p.kb) * (w.piece + 1) / split);
      w.slot = tl * (split - 1);
      return true;
    }
    return false;
  }
};

// Bytes one CTA's copies bring into a stage for work item w: A rows plus the CTA's B columns
// (64 instead of 128 for the half tile of a row-major B; a [N, K] B box is always 128 rows).
__device__ __forceinline__ uint32_t pair_half_bytes(const GemmParams& p, const PairWork& w) {
  return (w.half >= 0 && !p.b_trans) ? PR_A_STAGE + PR_B_STAGE / 2 : PR_STAGE_BYTES;
}

// The same for the pair's stage-load sequence number `seq` (walks the work list; abort path only).
__device__ uint32_t pair_seq_half_bytes(const GemmParams& p, int pair, int num_pairs, int seq) {
  PairIter it;
  it.init(p, pair);
  PairWork w;
  int base = 0;
  while (it.next(p, pair, num_pairs, w)) {
    if (seq < base + (w.k1 - w.k0)) return pair_half_bytes(p, w);
    base += w.k1 - w.k0;
  }
  return PR_STAGE_BYTES;
}

__device__ __forceinline__ void pair_abort(PairCtl* ctl, uint32_t code) {
  atomicCAS(&g_gemm_status, 0u, code);
  *reinterpret_cast<volatile int*>(&ctl->abort) = 1;
  st_cluster_s32(mapa_shared(smem_u32(&ctl->abort), cluster_ctarank() ^ 1u), 1);
}

__global__ void __launch_bounds__(THREADS, 1) gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_a,
                                                               const __grid_constant__ CUtensorMap tmap_b,
                                                               const GemmParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + PR_STAGES * PR_A_STAGE;
  PairCtl* ctl = reinterpret_cast<PairCtl*>(smem + PR_STAGES * PR_STAGE_BYTES);
  volatile int* abort_flag = &ctl->abort;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < PR_STAGES; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&ctl->acc_full[a], 1);
      mbar_init(&ctl->acc_empty[a], 8);
    }
    mbar_init(&ctl->drain, 1);
    mbar_init(&ctl->sk_stored, 4);
    mbar_init(&ctl->sk_read, 4);
    ctl->abort = 0;
    ctl->issued = 0;
    ctl->peer_issued = 0;
    fence_mbar_init();
    prefetch_tensormap(&tmap_a);
    prefetch_tensormap(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc_pair(&ctl->tmem_base, TMEM_COLS);
    tmem_relinquish_pair();
  }
  // Barriers initialised and TMEM allocated in both CTAs before any cross-CTA signal.
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = ctl->tmem_base;
  // Launched with programmatic stream serialization (no workspace): the setup above overlaps
  // the previous kernel on the stream; every global access (A, B, bias, C) comes after this.
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (elect_one_lane()) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      PairIter it;
      it.init(p, pair);
      PairWork w;
      while (it.next(p, pair, num_pairs, w)) {
        int mb, nb;
        tile_coords(w.tile, p.num_m, p.num_n, mb, nb);
        const int m0 = mb * PR_TILE_M + static_cast<int>(rank) * PR_BM;
        // Each CTA holds half of the tile's B columns: 128 of a full tile, 64 of a half tile
        // (a [N, K] B is fetched as a 128-row box either way; the MMA reads the first 64).
        const int n0 = w.half < 0 ? nb * BN + static_cast<int>(rank) * PR_BN_HALF
                                  : nb * BN + w.half * PR_BN_HALF + static_cast<int>(rank) * (PR_BN_HALF / 2);
        const uint32_t half_bytes = pair_half_bytes(p, w);
        const int b_boxes = w.half < 0 ? PR_BN_HALF / 64 : 1;  // 64-column boxes of a row-major B
        bool ok = true;
        for (int kb = w.k0; kb < w.k1; ++kb) {
          if (!mbar_wait_bounded(&ctl->empty[stage], phase ^ 1, p.wait_limit, abort_flag)) {
            if (!*abort_flag) pair_abort(ctl, NTL_STATUS_TMA_EMPTY_WAIT);
            ok = false;
            break;
          }
          const uint32_t full_addr = mapa_shared(smem_u32(&ctl->full[stage]), 0);
          if (rank == 0) mbar_arrive_expect_tx(&ctl->full[stage], 2 * half_bytes);
          uint8_t* a_dst = sA + stage * PR_A_STAGE;
          uint8_t* b_dst = sB + stage * PR_B_STAGE;
          tma_load_2d_pair(a_dst, &tmap_a, full_addr, kb * BK, m0);
          if (p.b_trans) {
            tma_load_2d_pair(b_dst, &tmap_b, full_addr, kb * BK, n0);
          } else {
            for (int i = 0; i < b_boxes; ++i)
              tma_load_2d_pair(b_dst + i * (64 * BK * 2), &tmap_b, full_addr, n0 + i * 64, kb * BK);
          }
          ++issued;
          if (++stage == PR_STAGES) stage = 0, phase ^= 1;
        }
        if (!ok) break;
      }
      if (rank == 0) ctl->issued = issued;
      else st_cluster_s32(mapa_shared(smem_u32(&ctl->peer_issued), 0), issued);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (rank 0)
    if (rank == 0 && elect_one_lane()) {
      const uint32_t idesc_full = umma_idesc_f16_f32(PR_TILE_M, BN, 0, p.b_trans ? 0 : 1);
      const uint32_t idesc_half = umma_idesc_f16_f32(PR_TILE_M, BN / 2, 0, p.b_trans ? 0 : 1);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int local = 0;
      PairIter it;
      it.init(p, pair);
      PairWork w;
      for (; ok && it.next(p, pair, num_pairs, w); ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait_bounded(&ctl->acc_empty[acc], acc_phase ^ 1, p.wait_limit, abort_flag)) {
          if (!*abort_flag) pair_abort(ctl, NTL_STATUS_ACC_EMPTY_WAIT);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        const uint32_t idesc = w.half < 0 ? idesc_full : idesc_half;
        for (int kb = w.k0; kb < w.k1; ++kb) {
          if (!mbar_wait_bounded(&ctl->full[stage], phase, p.wait_limit, abort_flag)) {
            if (!*abort_flag) pair_abort(ctl, NTL_STATUS_MMA_FULL_WAIT);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * PR_A_STAGE);
          const uint32_t b_addr = smem_u32(sB + stage * PR_B_STAGE);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t adesc = umma_desc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t bdesc = p.b_trans ? umma_desc_sw128(b_addr + k * 32, 16, 1024)
                                             : umma_desc_sw128(b_addr + k * 2048, 64 * BK * 2, 1024);
            tc_mma_f16_ss_pair(d_tmem, adesc, bdesc, idesc, (kb > w.k0 || k > 0) ? 1u : 0u);
          }
          tc_commit_pair_mc(&ctl->empty[stage], 0x3);
          if (++stage == PR_STAGES) stage = 0, phase ^= 1;
        }
        if (!ok) break;
        tc_commit_pair_mc(&ctl->acc_full[acc], 0x3);
      }
      // Every MMA issued retires before TMEM is freed.
      tc_commit_pair(&ctl->drain);
      if (!mbar_wait_bounded(&ctl->drain, 0, int64_t(1) << 24, nullptr))
        atomicCAS(&g_gemm_status, 0u, NTL_STATUS_DRAIN_WAIT);
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..5, both CTAs)
    const int quarter = warp & 3;
    const int r_local = quarter * 32 + lane;
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
    int local = 0;
    PairIter it;
    it.init(p, pair);
    PairWork w;
    const int split = static_cast<int>(p.sk_units);
    for (; it.next(p, pair, num_pairs, w); ++local) {
      int mb, nb;
      tile_coords(w.tile, p.num_m, p.num_n, mb, nb);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait_bounded(&ctl->acc_full[acc], acc_phase, p.wait_limit, abort_flag)) {
        if (!*abort_flag) pair_abort(ctl, NTL_STATUS_ACC_FULL_WAIT);
        break;
      }
      __syncwarp();
      tc_fence_after();
      const uint32_t acc_emp = mapa_shared(smem_u32(&ctl->acc_empty[acc]), 0);
      if (w.piece > 0) {
        // Contributor: raw partial sums of this CTA's 128 rows -> workspace slot, then its flag.
        // Slot layout [column quad][row][4]: a warp's float4 stores are 512 contiguous bytes.
        const int slot = (w.slot + w.piece - 1) * 2 + static_cast<int>(rank);
        float4* dst = reinterpret_cast<float4*>(p.ws + static_cast<size_t>(slot) * SK_SLOT_FLOATS) + r_local;
        for (int chunk = 0; chunk < BN / 32; ++chunk) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_lane + acc * BN + chunk * 32, r);
          tc_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            __stcg(dst + static_cast<size_t>(chunk * 8 + j / 4) * PR_BM,
                   make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]),
                               __uint_as_float(r[j + 3])));
        }
        __threadfence();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive_cluster(acc_emp);
          mbar_arrive(&ctl->sk_stored);
        }
        if (warp == 2 && lane == 0) {
          if (mbar_wait_bounded(&ctl->sk_stored, 0, p.wait_limit, abort_flag)) {
            __threadfence();
            atomicExch(p.flags + slot, 1u);
          } else if (!*abort_flag) {
            pair_abort(ctl, NTL_STATUS_ACC_FULL_WAIT);
          }
        }
        continue;
      }
      const bool finalise = w.k1 < p.kb;  // piece 0 of a split tile
      if (finalise) {
        bool ready = true;
        for (int pc = 1; pc < split && ready; ++pc) {
          if (lane == 0) ready = wait_flag(p.flags + (w.slot + pc - 1) * 2 + rank, p.wait_limit, abort_flag);
          ready = __shfl_sync(0xffffffffu, ready ? 1 : 0, 0) != 0;
        }
        if (!ready) {
          if (!*abort_flag) pair_abort(ctl, NTL_STATUS_ACC_FULL_WAIT);
          break;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->sk_read);
      }
      const int row = mb * PR_TILE_M + static_cast<int>(rank) * PR_BM + r_local;
      const bool row_ok = row < p.M;
      float* crow = p.c + static_cast<int64_t>(row) * p.N;
      const float row_bias = (p.bias_mode == NTL_BIAS_M && row_ok) ? __ldg(p.bias + row) : 0.0f;
      float* bias_s = reinterpret_cast<float*>(smem + PR_STAGES * PR_STAGE_BYTES + 1024) + (warp - 2) * BN;
      const int ncol0 = nb * BN + (w.half < 0 ? 0 : w.half * PR_BN_HALF);
      const int nchunks = (w.half < 0 ? BN : PR_BN_HALF) / 32;
      if (p.bias_mode == NTL_BIAS_N) stage_bias_n(p, ncol0, bias_s, lane);
      for (int chunk = 0; chunk < nchunks; ++chunk) {
        const int col0 = ncol0 + chunk * 32;
        if (col0 >= p.N) break;
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_lane + acc * BN + chunk * 32, r);
        tc_wait_ld();
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        if (finalise) {
          for (int pc = 1; pc < split; ++pc) {
            const int slot = (w.slot + pc - 1) * 2 + static_cast<int>(rank);
            const float4* part =
                reinterpret_cast<const float4*>(p.ws + static_cast<size_t>(slot) * SK_SLOT_FLOATS) + r_local;
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              const float4 q = __ldcg(part + static_cast<size_t>(chunk * 8 + j / 4) * PR_BM);
              v[j] += q.x, v[j + 1] += q.y, v[j + 2] += q.z, v[j + 3] += q.w;
            }
          }
        }
        if (!row_ok) continue;
        store_row_chunk(v, p, row, col0, crow, row_bias, bias_s + chunk * 32);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_emp);
      if (finalise && warp == 2 && lane == 0) {
        // Every epilogue warp has seen the flags: reset them for the next launch.
        if (mbar_wait_bounded(&ctl->sk_read, 0, p.wait_limit, abort_flag)) {
          for (int pc = 1; pc < split; ++pc) atomicExch(p.flags + (w.slot + pc - 1) * 2 + rank, 0u);
        } else if (!*abort_flag) {
          pair_abort(ctl, NTL_STATUS_ACC_FULL_WAIT);
        }
      }
    }
  }

  // ------------------------------------------------------------ teardown
  tc_fence_before();
  cluster_sync_all();
  if (rank == 0 && threadIdx.x == 0 && *abort_flag) {
    // Stage loads of either CTA may still be in flight; they all count on this CTA's `full`
    // barriers.  Sequences below min(issued) are armed for both halves; between the two
    // counts one half is missing: arm the odd CTA's half, or retire the half that will not
    // come.  Then wait each barrier's pending phase (the last PR_STAGES sequences cover
    // every load not yet consumed).
    const int own = ctl->issued, peer = ctl->peer_issued;
    const int hi = own > peer ? own : peer;
    for (int i = hi > PR_STAGES ? hi - PR_STAGES : 0; i < hi; ++i) {
      const int s = i % PR_STAGES;
      const uint32_t ph = static_cast<uint32_t>(i / PR_STAGES) & 1u;
      const uint32_t half_bytes = pair_seq_half_bytes(p, pair, num_pairs, i);
      if (i >= own) mbar_arrive_expect_tx(&ctl->full[s], half_bytes);
      else if (i >= peer) mbar_complete_tx(&ctl->full[s], half_bytes);
      if (!mbar_wait_bounded(&ctl->full[s], ph, int64_t(1) << 24, nullptr))
        atomicCAS(&g_gemm_status, 0u, NTL_STATUS_DRAIN_WAIT);
    }
  }
  cluster_sync_all();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, TMEM_COLS);
}

// ------------------------------------------------------------------ CUDA-core fallback
// 64x64 output tile per 256-thread CTA, 4x4 outputs per thread, K step 16; fp16 operands
// converted to fp32 in shared memory, fp32 FMA accumulation.  Used only for shapes the
// TMA path cannot address.
constexpr int FB_T = 64, FB_K = 16;

__global__ void __launch_bounds__(256) gemm_simt_kernel(const __half* __restrict__ A, const __half* __restrict__ B,
                                                        GemmParams p) {
  __shared__ float As[FB_K][FB_T + 4];
  __shared__ float Bs[FB_K][FB_T + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * FB_T, n0 = blockIdx.x * FB_T;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < p.K; k0 += FB_K) {
    for (int i = threadIdx.x; i < FB_T * FB_K; i += 256) {
      const int r = i / FB_K, kk = i % FB_K;
      const int m = m0 + r, k = k0 + kk;
      As[kk][r] = (m < p.M && k < p.K) ? __half2float(A[static_cast<int64_t>(m) * p.K + k]) : 0.0f;
      const int n = n0 + r;
      float bv = 0.0f;
      if (n < p.N && k < p.K)
        bv = __half2float(p.b_trans ? B[static_cast<int64_t>(n) * p.K + k] : B[static_cast<int64_t>(k) * p.N + n]);
      Bs[kk][r] = bv;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < FB_K; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i], b[i] = Bs[kk][tx * 4 + i];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    if (m >= p.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n >= p.N) continue;
      float b = 0.0f;
      if (p.bias_mode == NTL_BIAS_N) b = p.bias[n];
      else if (p.bias_mode == NTL_BIAS_MN) b = p.bias[static_cast<int64_t>(m) * p.N + n];
      else if (p.bias_mode == NTL_BIAS_M) b = p.bias[m];
      p.c[static_cast<int64_t>(m) * p.N + n] = epi(acc[i][j], p.alpha, b, p.relu, p.bias_mode);
    }
  }
}

// ------------------------------------------------------------------ host side

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

// 2-D fp16 tensor map over a row-major [rows, cols] matrix, box {box_cols, box_rows}.
int make_map_f16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_cols,
                 uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return ntl_fail(NTL_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return ntl_fail(NTL_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return NTL_OK;
}

// The dynamic shared-memory opt-in is a per-device function attribute: set it once per
// device (the first call on a device must not be inside a stream capture).
int ensure_smem_attr() {
  static std::atomic<uint64_t> done_mask{0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return ntl_fail(NTL_ERR_CUDA, "cudaGetDevice failed");
  const uint64_t bit = dev < 64 ? (uint64_t(1) << dev) : 0;
  if (bit && (done_mask.load(std::memory_order_acquire) & bit)) return NTL_OK;
  cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e != cudaSuccess) return ntl_fail(NTL_ERR_CUDA, "cudaFuncSetAttribute(gemm): %s", cudaGetErrorString(e));
  done_mask.fetch_or(bit, std::memory_order_release);
  return NTL_OK;
}

// The pair kernel's shared-memory opt-in and how many 2-CTA clusters fit on the device at
// once (its persistent grid), cached per device.
int pair_clusters(int* clusters_out) {
  static std::atomic<int> cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return ntl_fail(NTL_ERR_CUDA, "cudaGetDevice failed");
  if (dev >= 0 && dev < 64) {
    const int c = cached[dev].load(std::memory_order_acquire);
    if (c > 0) {
      *clusters_out = c;
      return NTL_OK;
    }
  }
  cudaError_t e = cudaFuncSetAttribute(gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, PR_SMEM_BYTES);
  if (e != cudaSuccess) return ntl_fail(NTL_ERR_CUDA, "cudaFuncSetAttribute(gemm pair): %s", cudaGetErrorString(e));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2, 1, 1);
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.dynamicSmemBytes = PR_SMEM_BYTES;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2, attr[0].val.clusterDim.y = 1, attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  e = cudaOccupancyMaxActiveClusters(&clusters, gemm_pair_kernel, &cfg);
  if (e != cudaSuccess || clusters < 1)
    return ntl_fail(NTL_ERR_CUDA, "cudaOccupancyMaxActiveClusters(gemm pair): %s", cudaGetErrorString(e));
  if (dev >= 0 && dev < 64) cached[dev].store(clusters, std::memory_order_release);
  *clusters_out = clusters;
  return NTL_OK;
}

// Work plan of the pair kernel.  With a workspace, the tiles of the last partial wave are
// split along K over the otherwise idle pairs (2 to 4 pieces of at least 4 k-blocks each).
struct PairPlan {
  int num_m, num_n, tiles, kb, pairs, dp_tiles, split, split_pairs, nar_pairs;
  size_t ws_bytes;
};

constexpr int PR_MAX_SPLIT = 4, PR_MIN_PIECE_KB = 4;

int make_pair_plan(int64_t M, int64_t N, int64_t K, bool split_tail, PairPlan* pl) {
  int clusters = 0;
  if (int rc = pair_clusters(&clusters)) return rc;
  pl->num_m = static_cast<int>((M + PR_TILE_M - 1) / PR_TILE_M);
  pl->num_n = static_cast<int>((N + BN - 1) / BN);
  const int64_t tiles = static_cast<int64_t>(pl->num_m) * pl->num_n;
  NTL_REQUIRE(tiles < (int64_t(1) << 31), NTL_ERR_UNSUPPORTED, "gemm: too many tiles");
  pl->tiles = static_cast<int>(tiles);
  pl->kb = static_cast<int>((K + BK - 1) / BK);
  pl->pairs = static_cast<int>(tiles < clusters ? tiles : clusters);
  pl->dp_tiles = pl->tiles;
  pl->split = 1;
  pl->split_pairs = 0;
  pl->nar_pairs = 0;
  pl->ws_bytes = 0;
  const int left = pl->tiles % clusters;
  if (!split_tail && left > 0 && 2 * left <= clusters) {
    // The partial wave's tiles become 2 x `left` half tiles on otherwise idle pairs (with
    // fewer tiles than half the pairs, every tile is split and twice as many pairs work).
    pl->pairs = pl->tiles > clusters ? clusters : 2 * left;
    pl->dp_tiles = pl->tiles - left;
    pl->nar_pairs = 2 * left;
    return NTL_OK;
  }
  if (split_tail && left > 0) {
    int split = clusters / left;
    if (split > PR_MAX_SPLIT) split = PR_MAX_SPLIT;
    while (split >= 2 && pl->kb / split < PR_MIN_PIECE_KB) --split;
    if (split >= 2 && static_cast<size_t>(left) * (split - 1) * 2 > kWsMaxSlots) split = 1;
    if (split >= 2) {
      pl->pairs = clusters;
      pl->dp_tiles = pl->tiles - left;
      pl->split = split;
      pl->split_pairs = left * split;
      const size_t slots = static_cast<size_t>(left) * (split - 1) * 2;  // one per CTA half
      pl->ws_bytes = kWsFlagBytes + slots * SK_SLOT_FLOATS * sizeof(float);
    }
  }
  return NTL_OK;
}

int gemm_pair_launch(const uint16_t* a, const uint16_t* b, GemmParams p, void* ws, size_t ws_bytes, bool split_tail,
                     cudaStream_t s) {
  PairPlan pl;
  if (int rc = make_pair_plan(p.M, p.N, p.K, split_tail, &pl)) return rc;
  if (pl.split > 1) {
    NTL_REQUIRE(ws != nullptr && ws_bytes >= pl.ws_bytes, NTL_ERR_INVALID,
                "gemm: workspace of %zu bytes needed, %zu given", pl.ws_bytes, ws_bytes);
    NTL_REQUIRE(ntl_aligned(ws, 16), NTL_ERR_ALIGNMENT, "gemm: workspace must be 16-byte aligned");
  }
  p.num_m = pl.num_m, p.num_n = pl.num_n, p.kb = pl.kb;
  p.dp_tiles = pl.dp_tiles;
  p.sk_ctas = pl.split_pairs;
  p.sk_units = pl.split;
  p.nar_pairs = pl.nar_pairs;
  p.ws = pl.split > 1 ? reinterpret_cast<float*>(static_cast<unsigned char*>(ws) + kWsFlagBytes) : nullptr;
  p.flags = pl.split > 1 ? static_cast<uint32_t*>(ws) : nullptr;
  CUtensorMap ma, mb;
  if (int rc = make_map_f16(&ma, a, p.M, p.K, BK, PR_BM)) return rc;
  if (p.b_trans) {
    if (int rc = make_map_f16(&mb, b, p.N, p.K, BK, PR_BN_HALF)) return rc;
  } else {
    if (int rc = make_map_f16(&mb, b, p.K, p.N, 64, BK)) return rc;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pl.pairs), 1, 1);
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.dynamicSmemBytes = PR_SMEM_BYTES;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2, attr[0].val.clusterDim.y = 1, attr[0].val.clusterDim.z = 1;
  // Without a workspace the kernel's setup may overlap the previous kernel (it waits with
  // pdl_wait before touching global memory); with one, the launch keeps plain stream order
  // behind whatever cleared the workspace's flags.
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pl.split > 1 ? 1 : 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_pair_kernel, ma, mb, p);
  ntl_note_launch();
  if (e != cudaSuccess) return ntl_fail(NTL_ERR_CUDA, "gemm (CTA-pair path) launch: %s", cudaGetErrorString(e));
  return ntl_check_launch("gemm (CTA-pair path) launch");
}

// Work plan for an M x N x K problem.  Stream-K applies only with a workspace.
struct Plan {
  int num_m, num_n, tiles, kb, grid, dp_tiles, sk_ctas;
  int64_t sk_units;
  size_t ws_bytes;
};

int make_plan(int64_t M, int64_t N, int64_t K, bool stream_k, Plan* pl) {
  int sms = 0;
  if (int rc = ntl_num_sms(&sms)) return rc;
  pl->num_m = static_cast<int>((M + BM - 1) / BM);
  pl->num_n = static_cast<int>((N + BN - 1) / BN);
  const int64_t tiles = static_cast<int64_t>(pl->num_m) * pl->num_n;
  NTL_REQUIRE(tiles < (int64_t(1) << 31), NTL_ERR_UNSUPPORTED, "gemm: too many tiles");
  pl->tiles = static_cast<int>(tiles);
  pl->kb = static_cast<int>((K + BK - 1) / BK);
  pl->grid = static_cast<int>(tiles < sms ? tiles : sms);
  pl->dp_tiles = pl->tiles;
  pl->sk_ctas = 0;
  pl->sk_units = 0;
  pl->ws_bytes = 0;
  if (stream_k && pl->tiles % sms != 0) {
    const int dp = (pl->tiles / sms) * sms;
    const int64_t units = static_cast<int64_t>(pl->tiles - dp) * pl->kb;
    const int64_t ctas = std::min<int64_t>(std::min<int64_t>(sms, units / SK_MIN_UNITS), kWsMaxSlots);
    if (ctas >= 2) {
      pl->grid = sms;
      pl->dp_tiles = dp;
      pl->sk_units = units;
      pl->sk_ctas = static_cast<int>(ctas);
      pl->ws_bytes = kWsFlagBytes + static_cast<size_t>(ctas) * SK_SLOT_FLOATS * sizeof(float);
    }
  }
  return NTL_OK;
}

int gemm_launch(const uint16_t* a, const uint16_t* b, float* c, const float* bias, int bias_mode, float alpha,
                int relu, int64_t M, int64_t N, int64_t K, int b_trans, void* ws, size_t ws_bytes, bool stream_k,
                cudaStream_t s) {
  NTL_REQUIRE(M >= 0 && N >= 0 && K >= 0, NTL_ERR_INVALID, "gemm: negative size");
  NTL_REQUIRE(M < (int64_t(1) << 31) && N < (int64_t(1) << 31) && K < (int64_t(1) << 31), NTL_ERR_UNSUPPORTED,
              "gemm: dimensions must be < 2^31");
  NTL_REQUIRE(bias_mode >= NTL_BIAS_NONE && bias_mode <= NTL_BIAS_M, NTL_ERR_INVALID, "gemm: bad bias_mode %d",
              bias_mode);
  NTL_REQUIRE(bias_mode == NTL_BIAS_NONE || bias != nullptr, NTL_ERR_INVALID, "gemm: bias_mode needs a bias pointer");
  if (M == 0 || N == 0) return NTL_OK;
  NTL_REQUIRE(c && (K == 0 || (a && b)), NTL_ERR_INVALID, "gemm: NULL pointer");
  GemmParams p;
  p.nar_pairs = 0;
  p.c = c;
  p.bias = bias;
  p.bias_mode = bias_mode;
  p.alpha = alpha;
  p.relu = relu ? 1 : 0;
  p.M = static_cast<int>(M), p.N = static_cast<int>(N), p.K = static_cast<int>(K);
  p.b_trans = b_trans ? 1 : 0;
  p.vec_store = (N % 4 == 0 && ntl_aligned(c, 16)) ? 1 : 0;
  p.vec_bias = (bias != nullptr && N % 4 == 0 && ntl_aligned(bias, 16)) ? 1 : 0;
  p.wait_limit = ntl_wait_limit();
  const bool tma_ok = K > 0 && K % 8 == 0 && (b_trans || N % 8 == 0) && ntl_aligned(a, 16) && ntl_aligned(b, 16);
  if (!tma_ok) {
    dim3 grid(static_cast<unsigned>((N + FB_T - 1) / FB_T), static_cast<unsigned>((M + FB_T - 1) / FB_T));
    NTL_REQUIRE(grid.y <= 65535, NTL_ERR_UNSUPPORTED, "gemm: M too large for the unaligned path");
    gemm_simt_kernel<<<grid, 256, 0, s>>>(reinterpret_cast<const __half*>(a), reinterpret_cast<const __half*>(b), p);
    ntl_note_launch();
    return ntl_check_launch("gemm (CUDA-core path) launch");
  }
  if (M > PR_BM) return gemm_pair_launch(a, b, p, ws, ws_bytes, stream_k, s);
  Plan pl;
  if (int rc = make_plan(M, N, K, stream_k, &pl)) return rc;
  if (pl.sk_ctas > 0) {
    NTL_REQUIRE(ws != nullptr && ws_bytes >= pl.ws_bytes, NTL_ERR_INVALID,
                "gemm: workspace of %zu bytes needed, %zu given", pl.ws_bytes, ws_bytes);
    NTL_REQUIRE(ntl_aligned(ws, 16), NTL_ERR_ALIGNMENT, "gemm: workspace must be 16-byte aligned");
  }
  p.num_m = pl.num_m, p.num_n = pl.num_n, p.kb = pl.kb;
  p.dp_tiles = pl.dp_tiles;
  p.sk_ctas = pl.sk_ctas;
  p.sk_units = pl.sk_units;
  p.ws = pl.sk_ctas > 0 ? reinterpret_cast<float*>(static_cast<unsigned char*>(ws) + kWsFlagBytes) : nullptr;
  p.flags = pl.sk_ctas > 0 ? static_cast<uint32_t*>(ws) : nullptr;
  CUtensorMap ma, mb;
  if (int rc = make_map_f16(&ma, a, M, K, BK, BM)) return rc;
  if (b_trans) {
    if (int rc = make_map_f16(&mb, b, N, K, BK, BN)) return rc;
  } else {
    if (int rc = make_map_f16(&mb, b, K, N, 64, BK)) return rc;
  }
  if (int rc = ensure_smem_attr()) return rc;
  if (pl.sk_ctas > 0) {
    gemm_tc_kernel<<<pl.grid, THREADS, SMEM_BYTES, s>>>(ma, mb, p);
  } else {
    // No workspace: the setup may overlap the previous kernel (see the pair launch).
    cudaError_t e = ntl_launch_pdl(gemm_tc_kernel, dim3(pl.grid), dim3(THREADS), SMEM_BYTES, s, ma, mb, p);
    if (e != cudaSuccess) {
      ntl_note_launch();
      return ntl_fail(NTL_ERR_CUDA, "gemm (tcgen05 path) launch: %s", cudaGetErrorString(e));
    }
  }
  ntl_note_launch();
  return ntl_check_launch("gemm (tcgen05 path) launch");
}

}  // namespace

uint32_t ntl_gemm_status_read(int clear) {
  uint32_t v = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemm_status, sizeof(v)) != cudaSuccess) return 0;
  if (clear) {
    uint32_t z = 0;
    cudaMemcpyToSymbol(g_gemm_status, &z, sizeof(z));
  }
  return v;
}

extern "C" int ntl_gemm_f16_f32(const uint16_t* a, const uint16_t* b, float* c, const float* bias, int bias_mode,
                                float alpha, int relu, int64_t M, int64_t N, int64_t K, int b_trans,
                                ntl_stream_t stream) {
  return gemm_launch(a, b, c, bias, bias_mode, alpha, relu, M, N, K, b_trans, nullptr, 0, false,
                     static_cast<cudaStream_t>(stream));
}

extern "C" int ntl_gemm_workspace_size(int64_t M, int64_t N, int64_t K, int b_trans, uint64_t* bytes_out) {
  NTL_REQUIRE(bytes_out != nullptr, NTL_ERR_INVALID, "gemm_workspace_size: bytes_out is NULL");
  NTL_REQUIRE(M >= 0 && N >= 0 && K >= 0, NTL_ERR_INVALID, "gemm_workspace_size: negative size");
  *bytes_out = 0;
  if (M == 0 || N == 0 || K == 0 || K % 8 != 0 || (!b_trans && N % 8 != 0)) return NTL_OK;
  if (M > PR_BM) {
    PairPlan pp;
    if (int rc = make_pair_plan(M, N, K, true, &pp)) return rc;
    *bytes_out = pp.ws_bytes;
    return NTL_OK;
  }
  Plan pl;
  if (int rc = make_plan(M, N, K, true, &pl)) return rc;
  *bytes_out = pl.ws_bytes;
  return NTL_OK;
}

extern "C" int ntl_gemm_f16_f32_ws(const uint16_t* a, const uint16_t* b, float* c, const float* bias, int bias_mode,
                                   float alpha, int relu, int64_t M, int64_t N, int64_t K, int b_trans,
                                   void* workspace, uint64_t workspace_bytes, ntl_stream_t stream) {
  return gemm_launch(a, b, c, bias, bias_mode, alpha, relu, M, N, K, b_trans, workspace, workspace_bytes, true,
                     static_cast<cudaStream_t>(stream));
}

// ----------------------------------------------------------------- allocation-free variant
//
// Some callers cannot allocate device memory for a workspace: a plugin host that hands a
// kernel only its tensors and a stream (the reference's TVM-FFI launch path, for one, has no
// workspace argument), or a runtime that runs with the device allocator switched off after
// start-up.  ntl_gemm_f16_f32_noalloc gives them the split-K GEMM with its scratch in a
// file-scope device array instead of a caller buffer.
//
// The array is a fixed 16 MiB that every GPU loading this library holds until the process
// exits.  Shapes whose plan needs more are rejected with NTL_ERR_UNSUPPORTED: split tails of
// the CTA-pair kernel (M > 128) need at most ~15 MB, but a one-SM stream-K plan for M <= 128
// can need up to 148 slots of 128 KB (128 x 25600 x 4096 needs ~19 MB).  All calls share the array: the flag words are cleared
// (cudaMemsetAsync on the caller's stream) before every launch, and calls that overlap on
// the GPU race on it.  Host code cannot pass the array's name to a kernel (on the host it
// is a stand-in, not a device address), so the first call on each device looks up its
// device address with cudaGetSymbolAddress while that device is current; make that first
// call before any stream capture.  The address is cached per device together with the id of
// the context it was looked up in; after cudaDeviceReset the primary context (and the
// module holding the array) is new, so the next call looks the address up again.  The
// flag clear is one 4 KB cudaMemsetAsync on the caller's stream, enqueued before the
// kernel (it is not a kernel of this library and is not counted by ntl_launch_count).
// Nothing here allocates.
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
static __device__ __align__(256) unsigned char g_gemm_noalloc_scratch[kNoAllocScratchBytes];

namespace {
std::mutex g_scratch_mu;
struct ScratchAddr {
  unsigned long long ctx_id;
  void* ptr;
};
ScratchAddr g_scratch[64] = {};

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

// Id of the calling thread's current context (0 when the driver cannot say).
unsigned long long current_context_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(fn);
    fn = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(fn);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current == nullptr || get_id == nullptr || get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return ntl_fail(NTL_ERR_CUDA, "cudaGetDevice failed");
  if (dev < 0 || dev >= 64) return ntl_fail(NTL_ERR_UNSUPPORTED, "gemm_noalloc: device index %d out of range", dev);
  // Make the device's primary context current (cudaSetDevice initialises it) so the id and
  // the symbol address below refer to the context the launch will use.
  if (cudaSetDevice(dev) != cudaSuccess) return ntl_fail(NTL_ERR_CUDA, "gemm_noalloc: cudaSetDevice failed");
  const unsigned long long ctx = current_context_id();
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  ScratchAddr& slot = g_scratch[dev];
  if (slot.ptr == nullptr || ctx == 0 || slot.ctx_id != ctx) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_gemm_noalloc_scratch);
    if (e != cudaSuccess || ptr == nullptr)
      return ntl_fail(NTL_ERR_CUDA, "gemm_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
    slot.ptr = ptr;
    slot.ctx_id = ctx;
  }
  *out = slot.ptr;
  return NTL_OK;
}
}  // namespace

extern "C" int ntl_gemm_f16_f32_noalloc(const uint16_t* a, const uint16_t* b, float* c, const float* bias,
                                        int bias_mode, float alpha, int relu, int64_t M, int64_t N, int64_t K,
                                        int b_trans, ntl_stream_t stream) {
  uint64_t need = 0;
  // The same test gemm_launch applies: operands TMA cannot address take the CUDA-core path,
  // which needs no scratch (and is then neither refused for size nor preceded by a clear).
  const bool tma_ok = K > 0 && K % 8 == 0 && (b_trans || N % 8 == 0) && ntl_aligned(a, 16) && ntl_aligned(b, 16);
  if (tma_ok) {
    if (int rc = ntl_gemm_workspace_size(M, N, K, b_trans, &need)) return rc;
  }
  NTL_REQUIRE(need <= kNoAllocScratchBytes, NTL_ERR_UNSUPPORTED,
              "gemm_noalloc: this shape needs %llu bytes of scratch, more than the %zu-byte static maximum "
              "(use ntl_gemm_f16_f32_ws with a caller workspace)",
              (unsigned long long)need, kNoAllocScratchBytes);
  void* scratch = nullptr;
  if (need > 0) {
    if (int rc = noalloc_scratch(&scratch)) return rc;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (need > 0) {
    // The flag block at the front of the workspace must start at zero.
    cudaError_t e = cudaMemsetAsync(scratch, 0, kWsFlagBytes, s);
    if (e != cudaSuccess) return ntl_fail(NTL_ERR_CUDA, "gemm_noalloc: clearing flags: %s", cudaGetErrorString(e));
  }
  return gemm_launch(a, b, c, bias, bias_mode, alpha, relu, M, N, K, b_trans, need > 0 ? scratch : nullptr,
                     need > 0 ? kNoAllocScratchBytes : 0, true, s);
}
