// Out-of-place transpose of a row-major fp32 [m, n] matrix into [n, m].
//
// Reference: examples/transpose.py:5-15 — per 32x32 tile, a shared-memory staging copy
// tile[i, j] = A[bx*32 + i, by*32 + j] followed by B[by*32 + i, bx*32 + j] = tile[j, i];
// elements outside A are neither read nor written.  The result is a bit-exact copy.
//
// Here each 256-thread CTA moves one 32x32 tile: every warp reads and writes whole
// 128-byte row segments (coalesced on both sides) through a 32 x 33 shared tile (the extra
// column puts the column reads of the transposed pass on 32 different banks).  Streaming
// loads and stores, and the same launch prologue as the row kernels: prefetch the tile's
// rows into L2, then wait for the previous kernel on the stream (programmatic dependent
// launch).
#include "ntl_common.cuh"

namespace {

constexpr int kTile = 32;
constexpr int kRowsPerPass = 8;  // blockDim = (32, 8)

__global__ void __launch_bounds__(kTile * kRowsPerPass) transpose_f32_kernel(const float* __restrict__ a,
                                                                             float* __restrict__ b, int64_t m,
                                                                             int64_t n) {
  __shared__ float tile[kTile][kTile + 1];
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * kTile;  // tile rows of A
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * kTile;  // tile columns of A
  const int tx = threadIdx.x, ty = threadIdx.y;
  if (tx == 0) {
    for (int k = ty; k < kTile; k += kRowsPerPass) {
      const int64_t r = r0 + k;
      if (r < m && c0 < n) prefetch_l2(a + r * n + c0, (n - c0 < kTile ? n - c0 : kTile) * 4);
    }
  }
  pdl_wait();
  pdl_trigger();
  const int64_t c = c0 + tx;
#pragma unroll
  for (int k = ty; k < kTile; k += kRowsPerPass) {
    const int64_t r = r0 + k;
    if (r < m && c < n) tile[k][tx] = __ldcs(a + r * n + c);
  }
  __syncthreads();
  const int64_t oc = r0 + tx;  // output column = input row
#pragma unroll
  for (int k = ty; k < kTile; k += kRowsPerPass) {
    const int64_t orow = c0 + k;  // output row = input column
    if (orow < n && oc < m) __stcs(b + orow * m + oc, tile[tx][k]);
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
  dim3 grid(static_cast<unsigned>(tiles_c), static_cast<unsigned>(tiles_r)), block(kTile, kRowsPerPass);
  ntl_launch_pdl(transpose_f32_kernel, grid, block, 0, static_cast<cudaStream_t>(stream), a, b, m, n);
  ntl_note_launch();
  return ntl_check_launch("transpose launch");
}
