// FlashAttention-2 forward on sm_100a: TMA + tcgen05 MMA with TMEM accumulators.
//
// Reference: the kernel its emitter builds for examples/flash_attention.py:26-79 — per
// (batch, head, 64-row query tile): S = Q K^T, online softmax in base 2 with
// scale = log2(e)/sqrt(d) (:23), causal fill -1e30 (:56-62), P cast to fp16 before P V
// (:74-75), O /= l at the end (:77-78); sm_80 mma.sync with smem round trips for the row
// statistics (codegen.py:972-984, :1062-1073).
//
// Design (one CTA = one (batch, head, 128-query tile); 192 threads):
//   warp 0      TMA: Q once, then K_j / V_j (128 keys x D) into a 2-stage ring.  3-D tensor
//               maps [B*H, S, D] so rows past S are zero-filled and never cross heads.
//   warp 1      TMEM owner (512 columns: S double buffer 2x128, O 128) and MMA issuer:
//               S_j = Q K_j^T (SS, K-major B) is issued before O += P_{j-1} V_{j-1} (SS,
//               P from smem, V N-major), so QK^T of the next tile overlaps the softmax.
//   warps 2..5  softmax, one query row per thread (TMEM lane = row): row max of S_j, then
//               p = exp2(s*c - m*c) into a double-buffered 128B-swizzled fp16 P tile,
//               l = l*r + sum(p), O *= r in TMEM once P V_{j-1} retired; final O / l -> fp16.
// Masked scores (causal key > query, keys >= S) contribute exactly 0 like the reference's
// -1e30 fill.  Every mbarrier wait is bounded; a wait that gives up records a status code,
// drains in-flight copies and MMAs, frees TMEM and returns.
#include <atomic>
#include <mutex>

#include "ntl_common.cuh"

namespace {

__device__ uint32_t g_fa2_status;

constexpr int BM = 128;  // query rows per CTA
constexpr int BN = 128;  // keys per KV tile
constexpr int THREADS = 192;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t S_COL = 0;    // S buffers at columns [0,128) and [128,256)
constexpr uint32_t O_COL = 256;  // O at [256, 256 + D)

struct Fa2Params {
  __half* o;
  int S, H, n_qt;
  int causal;
  float c;  // softmax scale in log2 units
  int64_t wait_limit;
};

struct __align__(8) Fa2Ctl {
  uint64_t q_full;
  uint64_t k_full[2], v_full[2], kv_empty[2];
  uint64_t s_full[2], s_free[2];
  uint64_t p_full;
  uint64_t o_done;
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

template <int D>
struct Fa2Smem {
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int P_BYTES = BM * BN * 2;
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + Q_BYTES;
  static constexpr int V_OFF = K_OFF + 2 * KV_BYTES;
  static constexpr int P_OFF = V_OFF + 2 * KV_BYTES;
  static constexpr int CTL_OFF = P_OFF + 2 * P_BYTES;
  static constexpr int USED = CTL_OFF + 256;
  // >= 116 KB keeps one CTA per SM, so the 512-column TMEM allocation never contends.
  static constexpr int BYTES = (USED + 1024 > 118784 ? USED + 1024 : 118784);
};

__device__ __forceinline__ void fa2_abort(Fa2Ctl* ctl, uint32_t code) {
  atomicCAS(&g_fa2_status, 0u, code);
  *reinterpret_cast<volatile int*>(&ctl->abort) = 1;
}

// Byte offset of 16-byte chunk `chunk` (0..7) of row `row` inside a 128B-swizzled atom
// column of 128-byte rows (the layout TMA SWIZZLE_128B writes and UMMA reads).
__device__ __forceinline__ uint32_t sw128_offset(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

template <int D>
__global__ void __launch_bounds__(THREADS, 1) fa2_fwd_kernel(const __grid_constant__ CUtensorMap tq,
                                                             const __grid_constant__ CUtensorMap tk,
                                                             const __grid_constant__ CUtensorMap tv,
                                                             const Fa2Params p) {
  using L = Fa2Smem<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Fa2Ctl* ctl = reinterpret_cast<Fa2Ctl*>(smem + L::CTL_OFF);
  volatile int* abort_flag = &ctl->abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Heavy causal tiles first: the last query tile has the most KV tiles.
  const int qt = p.causal ? (p.n_qt - 1 - static_cast<int>(blockIdx.x)) : static_cast<int>(blockIdx.x);
  const int h = blockIdx.y, b = blockIdx.z;
  const int bh = b * p.H + h;
  const int q0 = qt * BM;
  const int n_kv_all = (p.S + BN - 1) / BN;
  const int n_kv = p.causal ? min(n_kv_all, (q0 + BM - 1) / BN + 1) : n_kv_all;

  if (threadIdx.x == 0) {
    mbar_init(&ctl->q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&ctl->k_full[s], 1);
      mbar_init(&ctl->v_full[s], 1);
      mbar_init(&ctl->kv_empty[s], 1);
      mbar_init(&ctl->s_full[s], 1);
      mbar_init(&ctl->s_free[s], 4);
    }
    mbar_init(&ctl->p_full, 4);
    mbar_init(&ctl->o_done, 1);
    mbar_init(&ctl->drain, 1);
    ctl->abort = 0;
    fence_mbar_init();
    prefetch_tensormap(&tq);
    prefetch_tensormap(&tk);
    prefetch_tensormap(&tv);
  }
  if (warp == 1) {
    tmem_alloc(&ctl->tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (elect_one_lane()) {
      bool ok = true;
      int issued = 0;
      mbar_arrive_expect_tx(&ctl->q_full, L::Q_BYTES);
#pragma unroll
      for (int d = 0; d < D / 64; ++d) tma_load_3d(smem + L::Q_OFF + d * (BM * 128), &tq, &ctl->q_full, d * 64, q0, bh);
      for (int j = 0; j < n_kv && ok; ++j) {
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait_bounded(&ctl->kv_empty[s], ph ^ 1, p.wait_limit, abort_flag)) {
          if (!*abort_flag) fa2_abort(ctl, NTL_STATUS_TMA_EMPTY_WAIT);
          ok = false;
          break;
        }
        const int k0 = j * BN;
        mbar_arrive_expect_tx(&ctl->k_full[s], L::KV_BYTES);
#pragma unroll
        for (int d = 0; d < D / 64; ++d)
          tma_load_3d(smem + L::K_OFF + s * L::KV_BYTES + d * (BN * 128), &tk, &ctl->k_full[s], d * 64, k0, bh);
        mbar_arrive_expect_tx(&ctl->v_full[s], L::KV_BYTES);
#pragma unroll
        for (int d = 0; d < D / 64; ++d)
          tma_load_3d(smem + L::V_OFF + s * L::KV_BYTES + d * (BN * 128), &tv, &ctl->v_full[s], d * 64, k0, bh);
        ++issued;
      }
      if (!ok) {
        // Drain every copy this thread issued before the CTA exits.
        if (!mbar_wait_bounded(&ctl->q_full, 0, int64_t(1) << 24, nullptr))
          atomicCAS(&g_fa2_status, 0u, NTL_STATUS_DRAIN_WAIT);
        for (int j = max(0, issued - 2); j < issued; ++j) {
          const int s = j & 1;
          const uint32_t ph = (j >> 1) & 1;
          if (!mbar_wait_bounded(&ctl->k_full[s], ph, int64_t(1) << 24, nullptr) ||
              !mbar_wait_bounded(&ctl->v_full[s], ph, int64_t(1) << 24, nullptr))
            atomicCAS(&g_fa2_status, 0u, NTL_STATUS_DRAIN_WAIT);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (elect_one_lane()) {
      constexpr uint32_t idesc_s = umma_idesc_f16_f32(BM, BN, 0, 0);  // B = K tile, K-major
      constexpr uint32_t idesc_o = umma_idesc_f16_f32(BM, D, 0, 1);   // B = V tile, N-major
      bool ok = mbar_wait_bounded(&ctl->q_full, 0, p.wait_limit, abort_flag);
      if (!ok && !*abort_flag) fa2_abort(ctl, NTL_STATUS_MMA_FULL_WAIT);
      const uint32_t q_addr = smem_u32(smem + L::Q_OFF);
      auto issue_pv = [&](int j) -> bool {
        const int s = j & 1;
        if (!mbar_wait_bounded(&ctl->p_full, j & 1, p.wait_limit, abort_flag) ||
            !mbar_wait_bounded(&ctl->v_full[s], (j >> 1) & 1, p.wait_limit, abort_flag)) {
          if (!*abort_flag) fa2_abort(ctl, NTL_STATUS_MMA_FULL_WAIT);
          return false;
        }
        tc_fence_after();
        const uint32_t p_addr = smem_u32(smem + L::P_OFF + (j & 1) * L::P_BYTES);
        const uint32_t v_addr = smem_u32(smem + L::V_OFF + s * L::KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t adesc = umma_desc_sw128(p_addr + (kk >> 2) * (BM * 128) + (kk & 3) * 32, 16, 1024);
          const uint64_t bdesc = umma_desc_sw128(v_addr + kk * 2048, BN * 128, 1024);
          tc_mma_f16_ss(tmem + O_COL, adesc, bdesc, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(&ctl->o_done);
        tc_commit(&ctl->kv_empty[s]);
        return true;
      };
      for (int j = 0; j < n_kv && ok; ++j) {
        const int s = j & 1;
        if (!mbar_wait_bounded(&ctl->k_full[s], (j >> 1) & 1, p.wait_limit, abort_flag) ||
            (j >= 2 && !mbar_wait_bounded(&ctl->s_free[s], ((j >> 1) & 1) ^ 1, p.wait_limit, abort_flag))) {
          if (!*abort_flag) fa2_abort(ctl, NTL_STATUS_MMA_FULL_WAIT);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + L::K_OFF + s * L::KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
          const uint32_t koff = (kk >> 2) * (BN * 128) + (kk & 3) * 32;
          tc_mma_f16_ss(tmem + S_COL + s * BN, umma_desc_sw128(q_addr + off, 16, 1024),
                        umma_desc_sw128(k_addr + koff, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
        }
        tc_commit(&ctl->s_full[s]);
        if (j >= 1 && !issue_pv(j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok) ok = issue_pv(n_kv - 1);
      if (!ok) {
        tc_commit(&ctl->drain);
        if (!mbar_wait_bounded(&ctl->drain, 0, int64_t(1) << 24, nullptr))
          atomicCAS(&g_fa2_status, 0u, NTL_STATUS_DRAIN_WAIT);
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax warps
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // row in tile == TMEM lane
    const int qrow = q0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const float c = p.c;
    float m_old = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const int s = j & 1;
      const int k0 = j * BN;
      if (!mbar_wait_bounded(&ctl->s_full[s], (j >> 1) & 1, p.wait_limit, abort_flag)) {
        if (!*abort_flag) fa2_abort(ctl, NTL_STATUS_SOFTMAX_WAIT);
        ok = false;
        break;
      }
      __syncwarp();
      tc_fence_after();
      const uint32_t s_addr = tmem + lane_off + S_COL + s * BN;
      const bool masked_tile = (k0 + BN > p.S) || (p.causal && k0 + BN - 1 > q0);
      // pass 1: row max
      float mx = -INFINITY;
#pragma unroll
      for (int ch = 0; ch < BN / 32; ++ch) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(s_addr + ch * 32, v);
        tc_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int key = k0 + ch * 32 + e;
          const bool keep = !masked_tile || (key < p.S && (!p.causal || key <= qrow));
          mx = fmaxf(mx, keep ? __uint_as_float(v[e]) : -INFINITY);
        }
      }
      const float m_new = fmaxf(m_old, mx);
      const float mc = m_new * c;
      // pass 2: p = exp2(s*c - m*c) -> fp16 P tile (row r), running sum
      float sum = 0.0f;
      const uint32_t p_base = smem_u32(smem + L::P_OFF + s * L::P_BYTES);
#pragma unroll
      for (int ch = 0; ch < BN / 32; ++ch) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(s_addr + ch * 32, v);
        tc_wait_ld();
        float pv[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int key = k0 + ch * 32 + e;
          const bool keep = !masked_tile || (key < p.S && (!p.causal || key <= qrow));
          pv[e] = keep ? exp2f(__fmaf_rn(__uint_as_float(v[e]), c, -mc)) : 0.0f;
          sum += pv[e];
        }
        // 32 keys = 4 chunks of 8 halves; keys [64a, 64a+64) live in atom column a.
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int key_chunk = ch * 4 + q;  // 0..15 chunks of 8 keys
          const uint32_t addr = p_base + (key_chunk >> 3) * (BM * 128) + sw128_offset(r, key_chunk & 7);
          st_shared_v4(addr, pack_half2(pv[q * 8 + 0], pv[q * 8 + 1]), pack_half2(pv[q * 8 + 2], pv[q * 8 + 3]),
                       pack_half2(pv[q * 8 + 4], pv[q * 8 + 5]), pack_half2(pv[q * 8 + 6], pv[q * 8 + 7]));
        }
      }
      // S buffer s may now be overwritten by S_{j+2}.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->s_free[s]);
      const float rscale = (j == 0) ? 0.0f : exp2f(m_old * c - mc);
      l = (j == 0) ? sum : __fmaf_rn(l, rscale, sum);
      if (j > 0) {
        // O holds P_{<j} V; rescale it once P_{j-1} V_{j-1} has retired.
        if (!mbar_wait_bounded(&ctl->o_done, (j - 1) & 1, p.wait_limit, abort_flag)) {
          if (!*abort_flag) fa2_abort(ctl, NTL_STATUS_SOFTMAX_WAIT);
          ok = false;
          break;
        }
        __syncwarp();
        tc_fence_after();
        if (__any_sync(0xffffffffu, rscale != 1.0f)) {
#pragma unroll
          for (int ch = 0; ch < D / 16; ++ch) {
            uint32_t o[16];
            tmem_ld_32x32b_x16(tmem + lane_off + O_COL + ch * 16, o);
            tc_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * rscale);
            tmem_st_32x32b_x16(tmem + lane_off + O_COL + ch * 16, o);
          }
          tc_wait_st();
        }
      }
      fence_proxy_async_smem();  // P (generic-proxy stores) -> visible to the tensor core
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->p_full);
      m_old = m_new;
    }
    // epilogue: O / l -> fp16
    if (ok && mbar_wait_bounded(&ctl->o_done, (n_kv - 1) & 1, p.wait_limit, abort_flag)) {
      __syncwarp();
      tc_fence_after();
      const float inv_l = 1.0f / l;
      __half* orow = p.o + (static_cast<int64_t>(bh) * p.S + qrow) * D;
#pragma unroll
      for (int ch = 0; ch < D / 16; ++ch) {
        uint32_t o[16];
        tmem_ld_32x32b_x16(tmem + lane_off + O_COL + ch * 16, o);
        tc_wait_ld();
        if (qrow < p.S) {
          uint32_t h[8];
#pragma unroll
          for (int e = 0; e < 8; ++e)
            h[e] = pack_half2(__uint_as_float(o[2 * e]) * inv_l, __uint_as_float(o[2 * e + 1]) * inv_l);
          uint4* dst = reinterpret_cast<uint4*>(orow + ch * 16);
          dst[0] = make_uint4(h[0], h[1], h[2], h[3]);
          dst[1] = make_uint4(h[4], h[5], h[6], h[7]);
        }
      }
    } else if (ok && !*abort_flag) {
      fa2_abort(ctl, NTL_STATUS_SOFTMAX_WAIT);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
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

template <int D>
int launch_fa2(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const Fa2Params& p, int batch,
               int heads, cudaStream_t s) {
  static std::atomic<uint64_t> done_mask{0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return ntl_fail(NTL_ERR_CUDA, "cudaGetDevice failed");
  const uint64_t bit = dev < 64 ? (uint64_t(1) << dev) : 0;
  if (!(bit && (done_mask.load(std::memory_order_acquire) & bit))) {
    cudaError_t e = cudaFuncSetAttribute(fa2_fwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Fa2Smem<D>::BYTES);
    if (e != cudaSuccess) return ntl_fail(NTL_ERR_CUDA, "cudaFuncSetAttribute(fa2): %s", cudaGetErrorString(e));
    done_mask.fetch_or(bit, std::memory_order_release);
  }
  dim3 grid(static_cast<unsigned>(p.n_qt), static_cast<unsigned>(heads), static_cast<unsigned>(batch));
  fa2_fwd_kernel<D><<<grid, THREADS, Fa2Smem<D>::BYTES, s>>>(mq, mk, mv, p);
  ntl_note_launch();
  return ntl_check_launch("attention launch");
}

}  // namespace

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
  NTL_REQUIRE(heads <= 65535 && batch <= 65535, NTL_ERR_UNSUPPORTED, "attention: batch and heads must be <= 65535");
  CUtensorMap mq, mk, mv;
  const uint64_t bh = static_cast<uint64_t>(batch * heads);
  if (int rc = make_map_bshd(&mq, q, bh, seq, dim)) return rc;
  if (int rc = make_map_bshd(&mk, k, bh, seq, dim)) return rc;
  if (int rc = make_map_bshd(&mv, v, bh, seq, dim)) return rc;
  Fa2Params p;
  p.o = reinterpret_cast<__half*>(o);
  p.S = static_cast<int>(seq);
  p.H = static_cast<int>(heads);
  p.n_qt = static_cast<int>((seq + BM - 1) / BM);
  p.causal = causal ? 1 : 0;
  p.c = scale_log2;
  p.wait_limit = ntl_wait_limit();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dim == 64) return launch_fa2<64>(mq, mk, mv, p, static_cast<int>(batch), static_cast<int>(heads), s);
  return launch_fa2<128>(mq, mk, mv, p, static_cast<int>(batch), static_cast<int>(heads), s);
}
