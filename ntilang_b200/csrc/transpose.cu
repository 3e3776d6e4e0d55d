// Out-of-place transpose of a row-major fp32 [m, n] matrix into [n, m].
//
// Reference: examples/transpose.py:5-15 — per 32x32 tile, a shared-memory staging copy
// tile[i, j] = A[bx*32 + i, by*32 + j] followed by B[by*32 + i, bx*32 + j] = tile[j, i];
// elements outside A are neither read nor written.  The result is a bit-exact copy.
//
// Here each 256-thread CTA moves one 64x64 tile (16 KB in, 16 KB out): with 4 KB tiles the
// SM held too few bytes in flight to cover HBM latency (2.8 TB/s measured on B200 at
// 4096x4096, against 6.0 TB/s for this layout).  Each thread reads four 16-byte row
// segments of A and writes four 16-byte row segments of B (a warp covers two 256-byte row
// pieces per access), through a 64 x 65 shared tile whose extra column spreads the column
// reads of the transposed pass over the banks.  VEC_IN needs n % 4 == 0 and a 16-byte
// aligned A (every 4-column group is then wholly inside or outside the matrix); VEC_OUT the
// same for m and B; otherwise that side moves one element at a time with a bound check per
// element.  Streaming loads and stores; the CTA waits for the previous kernel on the stream
// (programmatic dependent launch) before its first load.  No L2 prefetch before that wait:
// with thousands of 32 KB tiles almost no CTA starts early, and the 64 prefetches per tile
// measured 5% slower (5.77 against 6.06 TB/s at 4096x4096).
#include "ntl_common.cuh"

namespace {

constexpr int kTile = 64;
constexpr int kThreads = 256;
constexpr int kQuads = kTile / 4;                // 16 four-column groups per tile row
constexpr int kRowsPerPass = kThreads / kQuads;  // 16

template <bool VEC_IN, bool VEC_OUT>
__global__ void __launch_bounds__(kThreads) transpose_f32_kernel(const float* __restrict__ a, float* __restrict__ b,
                                                                 int64_t m, int64_t n) {
  __shared__ float tile[kTile][kTile + 1];
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * kTile;  // tile rows of A
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * kTile;  // tile columns of A
  const int q = threadIdx.x % kQuads, rr = threadIdx.x / kQuads;
  pdl_wait();
  pdl_trigger();
#pragma unroll
  for (int k = rr; k < kTile; k += kRowsPerPass) {
    const int64_t r = r0 + k, c = c0 + 4 * q;
    float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (r < m) {
      if (VEC_IN) {
        if (c < n) {
          const float4 t = __ldcs(reinterpret_cast<const float4*>(a + r * n + c));
          v[0] = t.x, v[1] = t.y, v[2] = t.z, v[3] = t.w;
        }
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (c + e < n) v[e] = __ldcs(a + r * n + c + e);
      }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) tile[k][4 * q + e] = v[e];
  }
  __syncthreads();
#pragma unroll
  for (int k = rr; k < kTile; k += kRowsPerPass) {
    const int64_t orow = c0 + k, oc = r0 + 4 * q;  // output row = input column, output column = input row
    if (orow >= n) continue;
    float v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = tile[4 * q + e][k];
    if (VEC_OUT) {
      if (oc < m) __stcs(reinterpret_cast<float4*>(b + orow * m + oc), make_float4(v[0], v[1], v[2], v[3]));
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (oc + e < m) __stcs(b + orow * m + oc + e, v[e]);
    }
  }
}

}  // namespace

extern "C" int ntl_transpose_f32(const float* a, float* b, int64_t m, int64_t n, ntl_stream_t stream) {
  NTL_REQUIRE(m >= 0 && n >= 0, NTL_ERR_INVALID, "transpose: negative size");
  if (m == 0 || n == 0) return NTL_OK;
  NTL_REQUIRE(a && b, NTL_ERR_INVALID, "transpose: NULL pointer");
  NTL_REQUIRE(a != b, NTL_ERR_INVALID, "transpose: in-place transpose is not supported");
  const int64_t tiles_c = (n + kTile - 1) / kTile, tiles_r = (m + kTile - 1) / kTile;
  NTL_REQUIRE(tiles_c <= 0x7fffffff && tiles_r <= 65535, NTL_ERR_UNSUPPORTED,
              "transpose: matrix too large for the tile grid (%lld x %lld)", (long long)m, (long long)n);
  const dim3 grid(static_cast<unsigned>(tiles_c), static_cast<unsigned>(tiles_r)), block(kThreads);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool vin = (n % 4 == 0) && ntl_aligned(a, 16), vout = (m % 4 == 0) && ntl_aligned(b, 16);
  if (vin && vout) ntl_launch_pdl(transpose_f32_kernel<true, true>, grid, block, 0, s, a, b, m, n);
  else if (vin) ntl_launch_pdl(transpose_f32_kernel<true, false>, grid, block, 0, s, a, b, m, n);
  else if (vout) ntl_launch_pdl(transpose_f32_kernel<false, true>, grid, block, 0, s, a, b, m, n);
  else ntl_launch_pdl(transpose_f32_kernel<false, false>, grid, block, 0, s, a, b, m, n);
  ntl_note_launch();
  return ntl_check_launch("transpose launch");
}
