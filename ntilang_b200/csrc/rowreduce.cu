// Row reductions: softmax, RMSNorm and LayerNorm over [rows, cols] fp32.
//
// Reference (python/ntilang/codegen.py:1028-1240, examples/softmax.py:9-25,
// examples/rmsnorm.py:13-37): the tile row is padded to P = next_pow2(cols) with the op's
// padding value (-inf for softmax, 0 for RMSNorm), and row sums are a perfect binary tree
// over those P positions in column order: the warp shuffle-down tree over 32 consecutive
// columns followed by the pairwise tree over the 32-column groups (codegen.py:1094-1151).
//
// Layout here: lane l of a row's warp holds columns [128c + 4l, 128c + 4l + 4) for chunk
// c.  Position bits, low to high, are (element: 2 bits, lane: 5 bits, chunk), so the same
// perfect tree is: in-lane pairs (e0+e1)+(e2+e3), then xor-shuffle levels 1..16 (both lanes
// of a pair form the identical commutative sum), then pairwise over chunks.  Padding
// beyond cols contributes exact zeros (exp(-inf) = 0, 0^2 = 0), and t + 0 == t for the
// non-negative sums involved, so rounding to the next power of two of chunks is free.
// Maxima are order-independent (fmaxf).  One row is one warp; rows longer than 2048
// columns use one 256-thread CTA per row with the warp level of the tree in shared memory.
#include <math_constants.h>

#include "ntl_common.cuh"

namespace {

constexpr unsigned kFull = 0xffffffffu;
// Rows (warps) per block of the warp-per-row softmax, measured on B200 at 16384 x 512: 4 beat
// 2, 8 and 16.
constexpr int kSoftmaxWarpsPerBlock = 4;
// The RMSNorm warp kernel takes its rows per block (warps per block) at run time, sized so that
// two blocks per SM hold every row: ceil(rows / (2 * SMs)), clamped to 4..16 (wider rows: 16).
// At 4096 x 1024 on 148 SMs that is 14 rows: 0.885 of the copy bandwidth against 0.838 with
// 16-row blocks, whatever the register cap (graph-replayed launches, 6 interleaved repeats).
__host__ __device__ constexpr int rms_max_threads(int nch) { return nch <= 8 ? 1024 : 512; }
int rms_warps_per_block(int64_t rows, int64_t nch) {
  if (nch > 8) return 16;
  int sms = 0;
  if (ntl_num_sms(&sms) != NTL_OK || sms <= 0) return 16;
  const int64_t per_block = (rows + 2 * sms - 1) / (2 * sms);
  return static_cast<int>(per_block < 4 ? 4 : (per_block > 16 ? 16 : per_block));
}
// LayerNorm: 16 rows per block, two blocks per SM (4096 x 1024: 0.873 of the copy bandwidth against
// 0.82 with 14 rows and 0.80 with 8; unlike RMSNorm, which is fastest with 14) while the rows fill
// every SM with 16-row blocks; below that, ceil(rows / (2 * SMs)) rows per block (at least 4), so
// that a small launch still spreads over every SM (a 1024-row shard in 16-row blocks ran on 64 of
// 148 SMs).
constexpr int kLayernormWarpsPerBlock = 16;
int ln_warps_per_block(int64_t rows) {
  int sms = 0;
  if (ntl_num_sms(&sms) != NTL_OK || sms <= 0) return kLayernormWarpsPerBlock;
  if (rows >= int64_t(kLayernormWarpsPerBlock) * sms * 3 / 2) return kLayernormWarpsPerBlock;
  const int64_t per_block = (rows + 2 * sms - 1) / (2 * sms);
  return static_cast<int>(per_block < 4 ? 4 : (per_block > kLayernormWarpsPerBlock ? kLayernormWarpsPerBlock : per_block));
}

// Row loads: evict-first (STREAM) or default-cached.  The warp-per-row softmax, RMSNorm and
// LayerNorm kernels use default-cached loads (softmax +3%, RMSNorm and LayerNorm +4-6% together
// with the plain stores below, in graph-replayed back-to-back launches on B200).
//
// VEC (the dispatch guarantees cols % 4 == 0 and 16-byte aligned rows): a 4-column group is
// wholly inside or outside the row, so one predicate guards the float4 access.  A per-group
// bounds test with a scalar fallback path measured 14% slower at 4096 x 1024 (RMSNorm 7.0 vs
// 6.1 us per launch): the fallback branches kept the row's loads from issuing together.
template <bool VEC, bool STREAM = true>
__device__ __forceinline__ void load4(const float* __restrict__ row, int64_t col, int64_t cols, float pad,
                                      float (&v)[4]) {
  if (VEC) {
    float4 t = make_float4(pad, pad, pad, pad);
    const float4* p = reinterpret_cast<const float4*>(row + col);
    if (col < cols) t = STREAM ? __ldcs(p) : __ldg(p);
    v[0] = t.x, v[1] = t.y, v[2] = t.z, v[3] = t.w;
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = (col + e < cols) ? (STREAM ? __ldcs(row + col + e) : __ldg(row + col + e)) : pad;
  }
}

// Weights are read by every row: cached loads.
template <bool VEC>
__device__ __forceinline__ void load_w4(const float* __restrict__ w, int64_t col, int64_t cols, float (&v)[4]) {
  if (VEC) {
    float4 t = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (col < cols) t = __ldg(reinterpret_cast<const float4*>(w + col));
    v[0] = t.x, v[1] = t.y, v[2] = t.z, v[3] = t.w;
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = (col + e < cols) ? __ldg(w + col + e) : 0.0f;
  }
}

// Row stores: evict-first (STREAM) or plain write-back.  The warp-per-row softmax, RMSNorm and
// LayerNorm kernels measured 1-5% faster with plain stores in back-to-back launches: their
// output stays in L2 and is written back while the following launches read.
template <bool VEC, bool STREAM = true>
__device__ __forceinline__ void store4(float* __restrict__ row, int64_t col, int64_t cols, const float (&v)[4]) {
  if (VEC) {
    float4* p = reinterpret_cast<float4*>(row + col);
    const float4 t = make_float4(v[0], v[1], v[2], v[3]);
    if (col < cols) {
      if (STREAM) __stcs(p, t); else *p = t;
    }
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e)
      if (col + e < cols) {
        if (STREAM) __stcs(row + col + e, v[e]); else row[col + e] = v[e];
      }
  }
}

__device__ __forceinline__ float lane_pair_sum(const float (&v)[4]) {
  return __fadd_rn(__fadd_rn(v[0], v[1]), __fadd_rn(v[2], v[3]));
}

__device__ __forceinline__ float warp_tree_sum(float s) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) s = __fadd_rn(s, __shfl_xor_sync(kFull, s, o));
  return s;
}

__device__ __forceinline__ float warp_max(float m) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(kFull, m, o));
  return m;
}

// Perfect tree over N partial sums (N a power of two after implicit zero padding).
template <int N>
__device__ __forceinline__ float chunk_tree(float (&s)[N]) {
#pragma unroll
  for (int w = 1; w < N; w <<= 1) {
#pragma unroll
    for (int c = 0; c + w < N; c += 2 * w) s[c] = __fadd_rn(s[c], s[c + w]);
  }
  return s[0];
}

// ------------------------------------------------------------------------- softmax

template <int NCH, bool VEC>
__global__ void __launch_bounds__(kSoftmaxWarpsPerBlock * 32) softmax_rows_warp(const float* __restrict__ x,
                                                                         float* __restrict__ y, int64_t rows,
                                                                         int64_t cols) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kSoftmaxWarpsPerBlock + (threadIdx.x >> 5);
  if (lane == 0 && row < rows) prefetch_l2(x + row * cols, cols * 4);
  pdl_wait();
  pdl_trigger();
  if (row >= rows) return;
  const float* xr = x + row * cols;
  float* yr = y + row * cols;
  float v[NCH][4];
#pragma unroll
  for (int c = 0; c < NCH; ++c) load4<VEC, false>(xr, static_cast<int64_t>(c) * 128 + lane * 4, cols, -CUDART_INF_F, v[c]);
  float m = -CUDART_INF_F;
#pragma unroll
  for (int c = 0; c < NCH; ++c)
#pragma unroll
    for (int e = 0; e < 4; ++e) m = fmaxf(m, v[c][e]);
  m = warp_max(m);
  float s[NCH];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
#pragma unroll
    for (int e = 0; e < 4; ++e) v[c][e] = expf(__fsub_rn(v[c][e], m));
    s[c] = warp_tree_sum(lane_pair_sum(v[c]));
  }
  const float total = chunk_tree<NCH>(s);
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
#pragma unroll
    for (int e = 0; e < 4; ++e) v[c][e] = __fdiv_rn(v[c][e], total);
    store4<VEC, false>(yr, static_cast<int64_t>(c) * 128 + lane * 4, cols, v[c]);
  }
}

// One CTA (8 warps) per row; position bits (element 2, lane 5, warp 3, chunk).
template <int NCH, bool VEC>
__global__ void __launch_bounds__(256) softmax_rows_cta(const float* __restrict__ x, float* __restrict__ y,
                                                        int64_t rows, int64_t cols) {
  __shared__ float red[NCH][8];
  __shared__ float red_max[8];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t row = blockIdx.x;
  if (threadIdx.x == 0) prefetch_l2(x + row * cols, cols < 4096 ? cols * 4 : 16384);  // first 16 KB
  pdl_wait();
  pdl_trigger();
  const float* xr = x + row * cols;
  float* yr = y + row * cols;
  float v[NCH][4];
#pragma unroll
  for (int c = 0; c < NCH; ++c)
    load4<VEC>(xr, static_cast<int64_t>(c) * 1024 + threadIdx.x * 4, cols, -CUDART_INF_F, v[c]);
  float m = -CUDART_INF_F;
#pragma unroll
  for (int c = 0; c < NCH; ++c)
#pragma unroll
    for (int e = 0; e < 4; ++e) m = fmaxf(m, v[c][e]);
  m = warp_max(m);
  if (lane == 0) red_max[warp] = m;
  __syncthreads();
  m = red_max[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) m = fmaxf(m, red_max[w]);
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
#pragma unroll
    for (int e = 0; e < 4; ++e) v[c][e] = expf(__fsub_rn(v[c][e], m));
    float s = warp_tree_sum(lane_pair_sum(v[c]));
    if (lane == 0) red[c][warp] = s;
  }
  __syncthreads();
  float s[NCH];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    float t[8];
#pragma unroll
    for (int w = 0; w < 8; ++w) t[w] = red[c][w];
    s[c] = chunk_tree<8>(t);
  }
  const float total = chunk_tree<NCH>(s);
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
#pragma unroll
    for (int e = 0; e < 4; ++e) v[c][e] = __fdiv_rn(v[c][e], total);
    store4<VEC>(yr, static_cast<int64_t>(c) * 1024 + threadIdx.x * 4, cols, v[c]);
  }
}

// ------------------------------------------------------------------------- RMSNorm

template <int NCH, bool VEC>
__global__ void __launch_bounds__(rms_max_threads(NCH)) rmsnorm_rows_warp(const float* __restrict__ x,
                                                                         const float* __restrict__ w,
                                                                         float* __restrict__ y, int64_t rows,
                                                                         int64_t cols, float eps, float inv_n) {
  extern __shared__ float4 w_s4[];
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const bool live = row < rows;
  if (lane == 0 && live) prefetch_l2(x + row * cols, cols * 4);
  if (threadIdx.x == 32) prefetch_l2(w, cols * 4);
  pdl_wait();
  pdl_trigger();
  // gamma is staged in shared memory once per block, all of a thread's loads before its stores
  // (at most 4 float4: nq <= 512, at least 128 threads).  Read with __ldg chunk by chunk in the
  // epilogue, it cost each row a chain of L2 round trips at the end; with a different gamma per
  // call (a model's layers) staging measured 5.94 -> 5.70 us at 4096 x 1024 and 2.87 -> 2.38 us
  // at 512 rows.
  if (VEC) {
    const int nq = static_cast<int>(cols) >> 2;
    const int threads = static_cast<int>(blockDim.x);
    float4 tw[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = threadIdx.x + k * threads;
      if (i < nq) tw[k] = __ldg(reinterpret_cast<const float4*>(w) + i);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = threadIdx.x + k * threads;
      if (i < nq) w_s4[i] = tw[k];
    }
    for (int i = threadIdx.x + 4 * threads; i < nq; i += threads) w_s4[i] = __ldg(reinterpret_cast<const float4*>(w) + i);
  }
  const float* xr = x + row * cols;
  float* yr = y + row * cols;
  float v[NCH][4];
  if (live) {
#pragma unroll
    for (int c = 0; c < NCH; ++c) load4<VEC, false>(xr, static_cast<int64_t>(c) * 128 + lane * 4, cols, 0.0f, v[c]);
  }
  if (VEC) __syncthreads();
  if (!live) return;
  float s[NCH];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    float q[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) q[e] = __fmul_rn(v[c][e], v[c][e]);
    s[c] = warp_tree_sum(lane_pair_sum(q));
  }
  const float ss = chunk_tree<NCH>(s);
  const float inv = rsqrtf(__fadd_rn(__fmul_rn(ss, inv_n), eps));
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int64_t col = static_cast<int64_t>(c) * 128 + lane * 4;
    float wv[4];
    if (VEC) {
      float4 tw = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      if (col < cols) tw = w_s4[col >> 2];
      wv[0] = tw.x, wv[1] = tw.y, wv[2] = tw.z, wv[3] = tw.w;
    } else {
      load_w4<VEC>(w, col, cols, wv);
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) v[c][e] = __fmul_rn(__fmul_rn(v[c][e], inv), wv[e]);
    store4<VEC, false>(yr, col, cols, v[c]);
  }
}

template <int NCH, bool VEC>
__global__ void __launch_bounds__(256) rmsnorm_rows_cta(const float* __restrict__ x, const float* __restrict__ w,
                                                        float* __restrict__ y, int64_t rows, int64_t cols, float eps,
                                                        float inv_n) {
  __shared__ float red[NCH][8];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t row = blockIdx.x;
  if (threadIdx.x == 0) prefetch_l2(x + row * cols, cols < 4096 ? cols * 4 : 16384);  // first 16 KB
  if (threadIdx.x == 32) prefetch_l2(w, cols * 4);
  pdl_wait();
  pdl_trigger();
  const float* xr = x + row * cols;
  float* yr = y + row * cols;
  float v[NCH][4];
#pragma unroll
  for (int c = 0; c < NCH; ++c) load4<VEC>(xr, static_cast<int64_t>(c) * 1024 + threadIdx.x * 4, cols, 0.0f, v[c]);
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    float q[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) q[e] = __fmul_rn(v[c][e], v[c][e]);
    float s = warp_tree_sum(lane_pair_sum(q));
    if (lane == 0) red[c][warp] = s;
  }
  __syncthreads();
  float s[NCH];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    float t[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) t[k] = red[c][k];
    s[c] = chunk_tree<8>(t);
  }
  const float ss = chunk_tree<NCH>(s);
  const float inv = rsqrtf(__fadd_rn(__fmul_rn(ss, inv_n), eps));
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int64_t col = static_cast<int64_t>(c) * 1024 + threadIdx.x * 4;
    float wv[4];
    load_w4<VEC>(w, col, cols, wv);
#pragma unroll
    for (int e = 0; e < 4; ++e) v[c][e] = __fmul_rn(__fmul_rn(v[c][e], inv), wv[e]);
    store4<VEC>(yr, col, cols, v[c]);
  }
}

// ----------------------------------------------------------------------- LayerNorm
//
// examples/layernorm.py:18-43: mean = tree_sum(x) * inv_n; d = x - mean (0 in the padding);
// rstd = rsqrt(tree_sum(d * d) * inv_n + eps); y = ((d * rstd) * w) + b, every step rounded
// separately (no fused multiply-add), both sums perfect trees over the padded row.

template <int NCH>
__device__ __forceinline__ void centre(float (&v)[NCH][4], float mean, int64_t col0, int64_t stride, int64_t cols) {
#pragma unroll
  for (int c = 0; c < NCH; ++c)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int64_t col = col0 + static_cast<int64_t>(c) * stride + e;
      v[c][e] = col < cols ? __fsub_rn(v[c][e], mean) : 0.0f;
    }
}

// w and b are read by every row of the block: the block stages both in shared memory once
// (2 * cols floats) after the dependent-launch wait, so the epilogue reads them at shared-
// memory latency and the compiler does not hold 8 * NCH weight registers across the row.
// Up to 8 chunks the kernel is held to 64 registers (two 512-thread blocks per SM).  Rows are
// read with default-cached loads and written with plain stores (9% faster at 4096 x 1024 than
// evict-first hints, together with the predicated vector accesses of load4/store4).
// WPB: rows (warps) per block as a compile-time constant, or 0 to take it from blockDim.  The
// 16-row launch of full-size problems keeps the constant: reading it from blockDim measured 3%
// slower at 4096 x 1024, with the same registers and no spills.
template <int NCH, bool VEC, int WPB>
__device__ __forceinline__ void layernorm_rows_body(const float* __restrict__ x, const float* __restrict__ w,
                                                    const float* __restrict__ b, float* __restrict__ y,
                                                    int64_t rows, int64_t cols, float eps, float inv_n) {
  extern __shared__ float4 wb_s4[];  // w[cols] then b[cols]
  float* wb_s = reinterpret_cast<float*>(wb_s4);
  const int lane = threadIdx.x & 31;
  const int threads = WPB > 0 ? WPB * 32 : static_cast<int>(blockDim.x);
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (threads >> 5) + (threadIdx.x >> 5);
  const bool live = row < rows;
  if (lane == 0 && live) prefetch_l2(x + row * cols, cols * 4);
  if (threadIdx.x == 32) prefetch_l2(w, cols * 4);
  if (threadIdx.x == 64) prefetch_l2(b, cols * 4);
  pdl_wait();
  pdl_trigger();
  const int n = static_cast<int>(cols);  // <= 2048 on this path
  if (VEC && WPB > 0) {
    const int nq = n >> 2;
    for (int i = threadIdx.x; i < nq; i += threads) {
      wb_s4[i] = __ldg(reinterpret_cast<const float4*>(w) + i);
      wb_s4[nq + i] = __ldg(reinterpret_cast<const float4*>(b) + i);
    }
  } else if (VEC) {
    // Fewer threads per block: a thread stages up to 4 float4 of gamma and of beta (nq <= 512,
    // at least 128 threads).  All its loads go out before the first store, so a layer's weights
    // coming from DRAM cost one round trip, not one per iteration (1024 x 1024 with a cold
    // gamma/beta per call: 3.92 us staged one iteration at a time, against 3.60 us in 16-row
    // blocks that stage in one).
    constexpr int kMaxStage = 4;
    const int nq = n >> 2;
    float4 tw[kMaxStage], tb[kMaxStage];
#pragma unroll
    for (int k = 0; k < kMaxStage; ++k) {
      const int i = threadIdx.x + k * threads;
      if (i < nq) {
        tw[k] = __ldg(reinterpret_cast<const float4*>(w) + i);
        tb[k] = __ldg(reinterpret_cast<const float4*>(b) + i);
      }
    }
#pragma unroll
    for (int k = 0; k < kMaxStage; ++k) {
      const int i = threadIdx.x + k * threads;
      if (i < nq) {
        wb_s4[i] = tw[k];
        wb_s4[nq + i] = tb[k];
      }
    }
    for (int i = threadIdx.x + kMaxStage * threads; i < nq; i += threads) {  // none within the limits above
      wb_s4[i] = __ldg(reinterpret_cast<const float4*>(w) + i);
      wb_s4[nq + i] = __ldg(reinterpret_cast<const float4*>(b) + i);
    }
  } else {
    for (int i = threadIdx.x; i < n; i += threads) {
      wb_s[i] = __ldg(w + i);
      wb_s[n + i] = __ldg(b + i);
    }
  }
  const float* xr = x + row * cols;
  float v[NCH][4];
  if (live) {
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = c * 128 + lane * 4;
      if (VEC) {  // n % 4 == 0: a 4-column group is wholly inside or outside the row
        float4 t = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (col < n) t = __ldg(reinterpret_cast<const float4*>(xr + col));
        v[c][0] = t.x, v[c][1] = t.y, v[c][2] = t.z, v[c][3] = t.w;
      } else {
        load4<false, false>(xr, col, cols, 0.0f, v[c]);
      }
    }
  }
  __syncthreads();
  if (!live) return;
  float s[NCH];
#pragma unroll
  for (int c = 0; c < NCH; ++c) s[c] = warp_tree_sum(lane_pair_sum(v[c]));
  const float mean = __fmul_rn(chunk_tree<NCH>(s), inv_n);
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    float q[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      v[c][e] = (c * 128 + lane * 4 + e < n) ? __fsub_rn(v[c][e], mean) : 0.0f;
      q[e] = __fmul_rn(v[c][e], v[c][e]);
    }
    s[c] = warp_tree_sum(lane_pair_sum(q));
  }
  const float rstd = rsqrtf(__fadd_rn(__fmul_rn(chunk_tree<NCH>(s), inv_n), eps));
  float* yr = y + row * cols;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = c * 128 + lane * 4;
    if (col >= n) continue;
    float wv[4], bv[4];
    if (VEC) {
      const float4 tw = wb_s4[col >> 2], tb = wb_s4[(n + col) >> 2];
      wv[0] = tw.x, wv[1] = tw.y, wv[2] = tw.z, wv[3] = tw.w;
      bv[0] = tb.x, bv[1] = tb.y, bv[2] = tb.z, bv[3] = tb.w;
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        wv[e] = col + e < n ? wb_s[col + e] : 0.0f;
        bv[e] = col + e < n ? wb_s[n + col + e] : 0.0f;
      }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) v[c][e] = __fadd_rn(__fmul_rn(__fmul_rn(v[c][e], rstd), wv[e]), bv[e]);
    store4<VEC, false>(yr, col, cols, v[c]);
  }
}

template <int NCH, bool VEC>
__global__ void __launch_bounds__(kLayernormWarpsPerBlock * 32, (NCH <= 8 ? 2 : 1))
    layernorm_rows_warp(const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ b,
                        float* __restrict__ y, int64_t rows, int64_t cols, float eps, float inv_n) {
  layernorm_rows_body<NCH, VEC, kLayernormWarpsPerBlock>(x, w, b, y, rows, cols, eps, inv_n);
}

// The same with fewer rows per block (ln_warps_per_block below 16), taken from blockDim.
template <int NCH, bool VEC>
__global__ void __launch_bounds__(kLayernormWarpsPerBlock * 32, (NCH <= 8 ? 2 : 1))
    layernorm_rows_warp_n(const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ b,
                          float* __restrict__ y, int64_t rows, int64_t cols, float eps, float inv_n) {
  layernorm_rows_body<NCH, VEC, 0>(x, w, b, y, rows, cols, eps, inv_n);
}

// One CTA (8 warps) per row; position bits (element 2, lane 5, warp 3, chunk).
template <int NCH>
__device__ __forceinline__ float cta_tree_sum(float (&part)[NCH], float (*red)[8], int lane, int warp) {
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const float t = warp_tree_sum(part[c]);
    if (lane == 0) red[c][warp] = t;
  }
  __syncthreads();
  float s[NCH];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    float t[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) t[k] = red[c][k];
    s[c] = chunk_tree<8>(t);
  }
  __syncthreads();  // red is reused by the next sum
  return chunk_tree<NCH>(s);
}

template <int NCH, bool VEC>
__global__ void __launch_bounds__(256) layernorm_rows_cta(const float* __restrict__ x, const float* __restrict__ w,
                                                          const float* __restrict__ b, float* __restrict__ y,
                                                          int64_t rows, int64_t cols, float eps, float inv_n) {
  __shared__ float red[NCH][8];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t row = blockIdx.x;
  if (threadIdx.x == 0) prefetch_l2(x + row * cols, cols < 4096 ? cols * 4 : 16384);  // first 16 KB
  if (threadIdx.x == 32) prefetch_l2(w, cols * 4);
  if (threadIdx.x == 64) prefetch_l2(b, cols * 4);
  pdl_wait();
  pdl_trigger();
  const float* xr = x + row * cols;
  float* yr = y + row * cols;
  float v[NCH][4];
#pragma unroll
  for (int c = 0; c < NCH; ++c) load4<VEC>(xr, static_cast<int64_t>(c) * 1024 + threadIdx.x * 4, cols, 0.0f, v[c]);
  float part[NCH];
#pragma unroll
  for (int c = 0; c < NCH; ++c) part[c] = lane_pair_sum(v[c]);
  const float mean = __fmul_rn(cta_tree_sum<NCH>(part, red, lane, warp), inv_n);
  centre<NCH>(v, mean, threadIdx.x * 4, 1024, cols);
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    float q[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) q[e] = __fmul_rn(v[c][e], v[c][e]);
    part[c] = lane_pair_sum(q);
  }
  const float rstd = rsqrtf(__fadd_rn(__fmul_rn(cta_tree_sum<NCH>(part, red, lane, warp), inv_n), eps));
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int64_t col = static_cast<int64_t>(c) * 1024 + threadIdx.x * 4;
    float wv[4], bv[4];
    load_w4<VEC>(w, col, cols, wv);
    load_w4<VEC>(b, col, cols, bv);
#pragma unroll
    for (int e = 0; e < 4; ++e) v[c][e] = __fadd_rn(__fmul_rn(__fmul_rn(v[c][e], rstd), wv[e]), bv[e]);
    store4<VEC>(yr, col, cols, v[c]);
  }
}

// --------------------------------------------------------------------- dispatch

constexpr int64_t kMaxWarpCols = 2048;   // 16 chunks of 128 per warp
constexpr int64_t kMaxCtaCols = 16384;   // 16 chunks of 1024 per CTA

template <class WarpK, class CtaK>
struct Dispatch;

#define NTL_ROW_DISPATCH(KW, KC, VEC, WPB, WSMEM, ...)                                                         \
  do {                                                                                                  \
    const int64_t nch = (cols + 127) / 128;                                                             \
    if (cols <= kMaxWarpCols) {                                                                         \
      const int64_t blocks = (rows + (WPB)-1) / (WPB);                                                  \
      NTL_REQUIRE(blocks <= 0x7fffffff, NTL_ERR_UNSUPPORTED, "too many rows");                         \
      dim3 ntl_grid_(static_cast<unsigned>(blocks)), ntl_block_((WPB)*32);                                               \
      if (nch <= 1) ntl_launch_pdl(KW<1, VEC>, ntl_grid_, ntl_block_, (WSMEM), s, __VA_ARGS__);                                \
      else if (nch <= 2) ntl_launch_pdl(KW<2, VEC>, ntl_grid_, ntl_block_, (WSMEM), s, __VA_ARGS__);                           \
      else if (nch <= 4) ntl_launch_pdl(KW<4, VEC>, ntl_grid_, ntl_block_, (WSMEM), s, __VA_ARGS__);                           \
      else if (nch <= 8) ntl_launch_pdl(KW<8, VEC>, ntl_grid_, ntl_block_, (WSMEM), s, __VA_ARGS__);                           \
      else ntl_launch_pdl(KW<16, VEC>, ntl_grid_, ntl_block_, (WSMEM), s, __VA_ARGS__);                                        \
    } else {                                                                                            \
      NTL_REQUIRE(rows <= 0x7fffffff, NTL_ERR_UNSUPPORTED, "too many rows");                           \
      const int64_t cch = (cols + 1023) / 1024;                                                         \
      dim3 ntl_grid_(static_cast<unsigned>(rows)), ntl_block_(256);                                                      \
      if (cch <= 2) ntl_launch_pdl(KC<2, VEC>, ntl_grid_, ntl_block_, 0, s, __VA_ARGS__);                                \
      else if (cch <= 4) ntl_launch_pdl(KC<4, VEC>, ntl_grid_, ntl_block_, 0, s, __VA_ARGS__);                           \
      else if (cch <= 8) ntl_launch_pdl(KC<8, VEC>, ntl_grid_, ntl_block_, 0, s, __VA_ARGS__);                           \
      else ntl_launch_pdl(KC<16, VEC>, ntl_grid_, ntl_block_, 0, s, __VA_ARGS__);                                        \
    }                                                                                                   \
  } while (0)

}  // namespace

extern "C" int ntl_softmax_f32(const float* x, float* y, int64_t rows, int64_t cols, ntl_stream_t stream) {
  NTL_REQUIRE(rows >= 0 && cols >= 0, NTL_ERR_INVALID, "softmax: negative size");
  if (rows == 0 || cols == 0) return NTL_OK;
  NTL_REQUIRE(x && y, NTL_ERR_INVALID, "softmax: NULL pointer");
  NTL_REQUIRE(cols <= kMaxCtaCols, NTL_ERR_UNSUPPORTED, "softmax: rows longer than %lld columns are not supported",
              (long long)kMaxCtaCols);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool vec = (cols % 4 == 0) && ntl_aligned(x, 16) && ntl_aligned(y, 16);
  if (vec)
    NTL_ROW_DISPATCH(softmax_rows_warp, softmax_rows_cta, true, kSoftmaxWarpsPerBlock, 0, x, y, rows, cols);
  else
    NTL_ROW_DISPATCH(softmax_rows_warp, softmax_rows_cta, false, kSoftmaxWarpsPerBlock, 0, x, y, rows, cols);
  ntl_note_launch();
  return ntl_check_launch("softmax launch");
}

extern "C" int ntl_rmsnorm_f32(const float* x, const float* w, float* y, int64_t rows, int64_t cols, float eps,
                               float inv_n, ntl_stream_t stream) {
  NTL_REQUIRE(rows >= 0 && cols >= 0, NTL_ERR_INVALID, "rmsnorm: negative size");
  if (rows == 0 || cols == 0) return NTL_OK;
  NTL_REQUIRE(x && w && y, NTL_ERR_INVALID, "rmsnorm: NULL pointer");
  NTL_REQUIRE(cols <= kMaxCtaCols, NTL_ERR_UNSUPPORTED, "rmsnorm: rows longer than %lld columns are not supported",
              (long long)kMaxCtaCols);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool vec = (cols % 4 == 0) && ntl_aligned(x, 16) && ntl_aligned(y, 16) && ntl_aligned(w, 16);
  if (vec)
    NTL_ROW_DISPATCH(rmsnorm_rows_warp, rmsnorm_rows_cta, true, rms_warps_per_block(rows, nch), static_cast<size_t>(cols) * 4, x, w, y, rows, cols, eps, inv_n);
  else
    NTL_ROW_DISPATCH(rmsnorm_rows_warp, rmsnorm_rows_cta, false, rms_warps_per_block(rows, nch), static_cast<size_t>(cols) * 4, x, w, y, rows, cols, eps, inv_n);
  ntl_note_launch();
  return ntl_check_launch("rmsnorm launch");
}

extern "C" int ntl_layernorm_f32(const float* x, const float* w, const float* b, float* y, int64_t rows,
                                 int64_t cols, float eps, float inv_n, ntl_stream_t stream) {
  NTL_REQUIRE(rows >= 0 && cols >= 0, NTL_ERR_INVALID, "layernorm: negative size");
  if (rows == 0 || cols == 0) return NTL_OK;
  NTL_REQUIRE(x && w && b && y, NTL_ERR_INVALID, "layernorm: NULL pointer");
  NTL_REQUIRE(cols <= kMaxCtaCols, NTL_ERR_UNSUPPORTED, "layernorm: rows longer than %lld columns are not supported",
              (long long)kMaxCtaCols);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool vec = (cols % 4 == 0) && ntl_aligned(x, 16) && ntl_aligned(y, 16) && ntl_aligned(w, 16) &&
                   ntl_aligned(b, 16);
  const size_t wb_bytes = 2 * static_cast<size_t>(cols) * sizeof(float);  // warp path only: cols <= 2048
  const int wpb = ln_warps_per_block(rows);
  if (wpb == kLayernormWarpsPerBlock) {
    if (vec)
      NTL_ROW_DISPATCH(layernorm_rows_warp, layernorm_rows_cta, true, wpb, wb_bytes, x, w, b, y, rows, cols, eps,
                       inv_n);
    else
      NTL_ROW_DISPATCH(layernorm_rows_warp, layernorm_rows_cta, false, wpb, wb_bytes, x, w, b, y, rows, cols, eps,
                       inv_n);
  } else {
    if (vec)
      NTL_ROW_DISPATCH(layernorm_rows_warp_n, layernorm_rows_cta, true, wpb, wb_bytes, x, w, b, y, rows, cols, eps,
                       inv_n);
    else
      NTL_ROW_DISPATCH(layernorm_rows_warp_n, layernorm_rows_cta, false, wpb, wb_bytes, x, w, b, y, rows, cols, eps,
                       inv_n);
  }
  ntl_note_launch();
  return ntl_check_launch("layernorm launch");
}
