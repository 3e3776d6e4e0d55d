// Row-wise inclusive scans, forward or reverse, fp32: prefix sum (cumsum) and prefix maximum
// (cummax).
//
// Reference order (python/ntilang/scan.py:132-240 warp lowering, :349-389 evaluate):
// each row is cut into 32-column segments [32s, 32s+32) padded with +0; within a segment
// an inclusive Hillis-Steele scan runs with offsets 1, 2, 4, 8, 16 (new[p] = old[p] +
// old[p -/+ o]); then carries run sequentially: carry_first = +0 and
// carry_next = seg_local[last] + carry, and every output is local + carry.
//
// Layout here: one warp per row, a row chunk is 128 columns and lane l holds columns
// [128c + 4l, 128c + 4l + 4) as one float4, so a segment is 8 consecutive lanes.  The
// Hillis-Steele levels become in-lane adds plus __shfl_up/down by 1, 1, 1, 2, 4 lanes;
// the carry chain across the chunk's four segments is computed redundantly by every
// lane from the four segment totals.  Every add is the same IEEE fp32 add on the same two
// values as in the reference DAG (addition is commutative), so outputs are bit-identical.
//
// cummax runs the same DAG with max as the combine and -inf as the identity
// (scan.py:26-29): fmaxf ignores a NaN operand and orders +0 above -0, as the reference's
// evaluator does (scan.py:366-374), so the maximum is independent of the order too.
#include <math_constants.h>

#include "ntl_common.cuh"

namespace {

constexpr int kWarpsPerBlock = 4;
constexpr unsigned kFull = 0xffffffffu;

struct F4 {
  float v[4];
};

struct SumOp {
  static __device__ __forceinline__ float combine(float a, float b) { return __fadd_rn(a, b); }
  static __device__ __forceinline__ float identity() { return 0.0f; }
};
struct MaxOp {
  static __device__ __forceinline__ float combine(float a, float b) { return fmaxf(a, b); }
  static __device__ __forceinline__ float identity() { return -CUDART_INF_F; }
};

// Load one 4-column group; out-of-range columns read as the scan identity.  Loads and stores use
// the default caching (2.8% faster at 32768x256 than evict-first hints).  VEC (cols % 4 == 0,
// 16-byte aligned rows): a group is wholly inside or outside the row, so one predicate guards
// the float4 access instead of a bounds test with a scalar fallback path.
template <class Op, bool VEC>
__device__ __forceinline__ F4 load4(const float* __restrict__ row, int64_t col, int64_t cols) {
  F4 r;
  if (VEC) {
    const float id = Op::identity();
    float4 t = make_float4(id, id, id, id);
    if (col < cols) t = __ldg(reinterpret_cast<const float4*>(row + col));
    r.v[0] = t.x, r.v[1] = t.y, r.v[2] = t.z, r.v[3] = t.w;
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e) r.v[e] = (col + e < cols) ? __ldg(row + col + e) : Op::identity();
  }
  return r;
}

template <bool VEC>
__device__ __forceinline__ void store4(float* __restrict__ row, int64_t col, int64_t cols, const F4& r) {
  if (VEC) {
    if (col < cols) *reinterpret_cast<float4*>(row + col) = make_float4(r.v[0], r.v[1], r.v[2], r.v[3]);
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e)
      if (col + e < cols) row[col + e] = r.v[e];
  }
}

// In-segment inclusive Hillis-Steele scan, forward (towards higher columns).
// q = lane index inside the 8-lane segment.
template <class Op>
__device__ __forceinline__ void segment_scan_fwd(F4& x, int q) {
  // o = 1
  {
    float p3 = __shfl_up_sync(kFull, x.v[3], 1);
    float n3 = Op::combine(x.v[3], x.v[2]), n2 = Op::combine(x.v[2], x.v[1]), n1 = Op::combine(x.v[1], x.v[0]);
    float n0 = q >= 1 ? Op::combine(x.v[0], p3) : x.v[0];
    x.v[0] = n0, x.v[1] = n1, x.v[2] = n2, x.v[3] = n3;
  }
  // o = 2
  {
    float p2 = __shfl_up_sync(kFull, x.v[2], 1), p3 = __shfl_up_sync(kFull, x.v[3], 1);
    float n3 = Op::combine(x.v[3], x.v[1]), n2 = Op::combine(x.v[2], x.v[0]);
    float n1 = q >= 1 ? Op::combine(x.v[1], p3) : x.v[1];
    float n0 = q >= 1 ? Op::combine(x.v[0], p2) : x.v[0];
    x.v[0] = n0, x.v[1] = n1, x.v[2] = n2, x.v[3] = n3;
  }
  // o = 4, 8, 16: whole lanes 1, 2, 4 below
#pragma unroll
  for (int d = 1; d <= 4; d <<= 1) {
    float p[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) p[e] = __shfl_up_sync(kFull, x.v[e], d);
    if (q >= d) {
#pragma unroll
      for (int e = 0; e < 4; ++e) x.v[e] = Op::combine(x.v[e], p[e]);
    }
  }
}

// Reverse direction (towards lower columns): new[p] = old[p] + old[p + o] for p < 32 - o.
template <class Op>
__device__ __forceinline__ void segment_scan_rev(F4& x, int q) {
  {
    float n0 = __shfl_down_sync(kFull, x.v[0], 1);
    float m0 = Op::combine(x.v[0], x.v[1]), m1 = Op::combine(x.v[1], x.v[2]), m2 = Op::combine(x.v[2], x.v[3]);
    float m3 = q <= 6 ? Op::combine(x.v[3], n0) : x.v[3];
    x.v[0] = m0, x.v[1] = m1, x.v[2] = m2, x.v[3] = m3;
  }
  {
    float n0 = __shfl_down_sync(kFull, x.v[0], 1), n1 = __shfl_down_sync(kFull, x.v[1], 1);
    float m0 = Op::combine(x.v[0], x.v[2]), m1 = Op::combine(x.v[1], x.v[3]);
    float m2 = q <= 6 ? Op::combine(x.v[2], n0) : x.v[2];
    float m3 = q <= 6 ? Op::combine(x.v[3], n1) : x.v[3];
    x.v[0] = m0, x.v[1] = m1, x.v[2] = m2, x.v[3] = m3;
  }
#pragma unroll
  for (int d = 1; d <= 4; d <<= 1) {
    float p[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) p[e] = __shfl_down_sync(kFull, x.v[e], d);
    if (q + d <= 7) {
#pragma unroll
      for (int e = 0; e < 4; ++e) x.v[e] = Op::combine(x.v[e], p[e]);
    }
  }
}

// Scan one 128-column chunk held as F4 per lane, given the running carry; returns the
// carry out of the chunk.  Segment totals sit in lane 8s+7 element 3 (forward) or lane
// 8s element 0 (reverse).
template <class Op, bool REV>
__device__ __forceinline__ float scan_chunk(F4& x, float carry, int lane) {
  const int q = lane & 7;
  const int seg = lane >> 3;
  if (!REV) {
    segment_scan_fwd<Op>(x, q);
    float t0 = __shfl_sync(kFull, x.v[3], 7), t1 = __shfl_sync(kFull, x.v[3], 15);
    float t2 = __shfl_sync(kFull, x.v[3], 23), t3 = __shfl_sync(kFull, x.v[3], 31);
    float c0 = carry, c1 = Op::combine(t0, c0), c2 = Op::combine(t1, c1), c3 = Op::combine(t2, c2);
    float mine = seg == 0 ? c0 : seg == 1 ? c1 : seg == 2 ? c2 : c3;
#pragma unroll
    for (int e = 0; e < 4; ++e) x.v[e] = Op::combine(x.v[e], mine);
    return Op::combine(t3, c3);
  } else {
    segment_scan_rev<Op>(x, q);
    float t0 = __shfl_sync(kFull, x.v[0], 0), t1 = __shfl_sync(kFull, x.v[0], 8);
    float t2 = __shfl_sync(kFull, x.v[0], 16), t3 = __shfl_sync(kFull, x.v[0], 24);
    float c3 = carry, c2 = Op::combine(t3, c3), c1 = Op::combine(t2, c2), c0 = Op::combine(t1, c1);
    float mine = seg == 0 ? c0 : seg == 1 ? c1 : seg == 2 ? c2 : c3;
#pragma unroll
    for (int e = 0; e < 4; ++e) x.v[e] = Op::combine(x.v[e], mine);
    return Op::combine(t0, c0);
  }
}

// Rows of at most NCH*128 columns: all chunks of a row are loaded before any is scanned.
template <class Op, int NCH, bool REV, bool VEC>
__global__ void __launch_bounds__(kWarpsPerBlock * 32) scan_rows_reg(const float* __restrict__ x,
                                                                       float* __restrict__ y, int64_t rows,
                                                                       int64_t cols) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  if (lane == 0 && row < rows) prefetch_l2(x + row * cols, cols * 4);
  pdl_wait();
  pdl_trigger();
  if (row >= rows) return;
  const float* xr = x + row * cols;
  float* yr = y + row * cols;
  F4 v[NCH];
#pragma unroll
  for (int c = 0; c < NCH; ++c) v[c] = load4<Op, VEC>(xr, static_cast<int64_t>(c) * 128 + lane * 4, cols);
  // Chunks entirely beyond the last 32-column segment of the row are skipped: the
  // reference has no such segments (their identity totals would not change a carry anyway).
  const int nch = static_cast<int>((cols + 127) / 128);
  float carry = Op::identity();
  if (!REV) {
#pragma unroll
    for (int c = 0; c < NCH; ++c)
      if (c < nch) carry = scan_chunk<Op, false>(v[c], carry, lane);
  } else {
#pragma unroll
    for (int c = NCH - 1; c >= 0; --c)
      if (c < nch) carry = scan_chunk<Op, true>(v[c], carry, lane);
  }
#pragma unroll
  for (int c = 0; c < NCH; ++c)
    if (c < nch) store4<VEC>(yr, static_cast<int64_t>(c) * 128 + lane * 4, cols, v[c]);
}

// Long rows: groups of G chunks are loaded, scanned and stored in row order (or reverse).
template <class Op, bool REV, bool VEC>
__global__ void __launch_bounds__(kWarpsPerBlock * 32) scan_rows_loop(const float* __restrict__ x,
                                                                        float* __restrict__ y, int64_t rows,
                                                                        int64_t cols) {
  constexpr int G = 8;
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  if (lane == 0 && row < rows) prefetch_l2(x + row * cols, 4096);  // the first group of chunks
  pdl_wait();
  pdl_trigger();
  if (row >= rows) return;
  const float* xr = x + row * cols;
  float* yr = y + row * cols;
  const int64_t nch = (cols + 127) / 128;
  const int64_t ngroups = (nch + G - 1) / G;
  float carry = Op::identity();
  for (int64_t gi = 0; gi < ngroups; ++gi) {
    const int64_t g = REV ? (ngroups - 1 - gi) : gi;
    F4 v[G];
#pragma unroll
    for (int c = 0; c < G; ++c) v[c] = load4<Op, VEC>(xr, (g * G + c) * 128 + lane * 4, cols);
    if (!REV) {
#pragma unroll
      for (int c = 0; c < G; ++c)
        if (g * G + c < nch) carry = scan_chunk<Op, false>(v[c], carry, lane);
    } else {
#pragma unroll
      for (int c = G - 1; c >= 0; --c)
        if (g * G + c < nch) carry = scan_chunk<Op, true>(v[c], carry, lane);
    }
#pragma unroll
    for (int c = 0; c < G; ++c)
      if (g * G + c < nch) store4<VEC>(yr, (g * G + c) * 128 + lane * 4, cols, v[c]);
  }
}

template <class Op, bool REV, bool VEC>
int launch(const float* x, float* y, int64_t rows, int64_t cols, cudaStream_t s, const char* what) {
  const int64_t blocks = (rows + kWarpsPerBlock - 1) / kWarpsPerBlock;
  NTL_REQUIRE(blocks <= 0x7fffffff, NTL_ERR_UNSUPPORTED, "%s: too many rows (%lld)", what, (long long)rows);
  dim3 grid(static_cast<unsigned>(blocks)), block(kWarpsPerBlock * 32);
  const int64_t nch = (cols + 127) / 128;
  if (nch <= 1)
    ntl_launch_pdl(scan_rows_reg<Op, 1, REV, VEC>, grid, block, 0, s, x, y, rows, cols);
  else if (nch <= 2)
    ntl_launch_pdl(scan_rows_reg<Op, 2, REV, VEC>, grid, block, 0, s, x, y, rows, cols);
  else if (nch <= 4)
    ntl_launch_pdl(scan_rows_reg<Op, 4, REV, VEC>, grid, block, 0, s, x, y, rows, cols);
  else if (nch <= 8)
    ntl_launch_pdl(scan_rows_reg<Op, 8, REV, VEC>, grid, block, 0, s, x, y, rows, cols);
  else
    ntl_launch_pdl(scan_rows_loop<Op, REV, VEC>, grid, block, 0, s, x, y, rows, cols);
  ntl_note_launch();
  return ntl_check_launch(what);
}

template <class Op>
int scan_rows(const float* x, float* y, int64_t rows, int64_t cols, int reverse, ntl_stream_t stream,
              const char* what) {
  NTL_REQUIRE(rows >= 0 && cols >= 0, NTL_ERR_INVALID, "%s: negative size (%lld, %lld)", what, (long long)rows,
              (long long)cols);
  if (rows == 0 || cols == 0) return NTL_OK;
  NTL_REQUIRE(x && y, NTL_ERR_INVALID, "%s: NULL pointer", what);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool vec = (cols % 4 == 0) && ntl_aligned(x, 16) && ntl_aligned(y, 16);
  if (reverse)
    return vec ? launch<Op, true, true>(x, y, rows, cols, s, what) : launch<Op, true, false>(x, y, rows, cols, s, what);
  return vec ? launch<Op, false, true>(x, y, rows, cols, s, what) : launch<Op, false, false>(x, y, rows, cols, s, what);
}

}  // namespace

extern "C" int ntl_cumsum_f32(const float* x, float* y, int64_t rows, int64_t cols, int reverse,
                              ntl_stream_t stream) {
  return scan_rows<SumOp>(x, y, rows, cols, reverse, stream, "cumsum");
}

extern "C" int ntl_cummax_f32(const float* x, float* y, int64_t rows, int64_t cols, int reverse,
                              ntl_stream_t stream) {
  return scan_rows<MaxOp>(x, y, rows, cols, reverse, stream, "cummax");
}
