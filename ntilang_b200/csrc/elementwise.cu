// Elementwise fp32 binary ops (vector add and friends).
//
// Reference: the elementwise kernel its emitter produces for examples/vector_add.py:5-10
// computes one scalar IEEE add per element with one element per thread
// (codegen.py:1494-1517, :1694-1734).  Here each thread streams four float4 per
// iteration: 128-bit coalesced loads that bypass L1 allocation (the data is read once),
// streaming stores, and a grid sized as whole waves of the SM count.  Arithmetic is the
// same single fp32 op per element, so results are bit-identical.
#include "ntl_common.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;  // float4 per thread per iteration

template <int OP>
__device__ __forceinline__ float apply(float a, float b) {
  if constexpr (OP == 0) return __fadd_rn(a, b);
  if constexpr (OP == 1) return __fsub_rn(a, b);
  return __fmul_rn(a, b);
}

template <int OP>
__device__ __forceinline__ float4 apply4(float4 a, float4 b) {
  return make_float4(apply<OP>(a.x, b.x), apply<OP>(a.y, b.y), apply<OP>(a.z, b.z), apply<OP>(a.w, b.w));
}

// Vector path: every pointer 16-byte aligned.  n4 = n / 4 float4 elements; the scalar
// tail (n % 4) is handled by block 0.
template <int OP>
__global__ void __launch_bounds__(kThreads) binary_f32_v4(const float4* __restrict__ a, const float4* __restrict__ b,
                                                          float4* __restrict__ c, int64_t n4,
                                                          const float* __restrict__ at, const float* __restrict__ bt,
                                                          float* __restrict__ ct, int tail) {
  pdl_wait();
  pdl_trigger();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads * kUnroll;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * kThreads * kUnroll + threadIdx.x; base < n4;
       base += stride) {
    float4 va[kUnroll], vb[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      int64_t i = base + static_cast<int64_t>(u) * kThreads;
      if (i < n4) {
        va[u] = __ldcs(a + i);
        vb[u] = __ldcs(b + i);
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      int64_t i = base + static_cast<int64_t>(u) * kThreads;
      if (i < n4) __stcs(c + i, apply4<OP>(va[u], vb[u]));
    }
  }
  if (blockIdx.x == 0 && threadIdx.x < tail) ct[threadIdx.x] = apply<OP>(at[threadIdx.x], bt[threadIdx.x]);
}

// Scalar path for unaligned pointers.
template <int OP>
__global__ void __launch_bounds__(kThreads) binary_f32_scalar(const float* __restrict__ a,
                                                              const float* __restrict__ b, float* __restrict__ c,
                                                              int64_t n) {
  pdl_wait();
  pdl_trigger();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < n; i += stride)
    c[i] = apply<OP>(__ldcs(a + i), __ldcs(b + i));
}

template <int OP>
int launch_binary(const float* a, const float* b, float* c, int64_t n, cudaStream_t stream) {
  int sms = 0;
  if (int rc = ntl_num_sms(&sms)) return rc;
  const int64_t max_blocks = static_cast<int64_t>(sms) * 8;  // 8 resident 256-thread CTAs per SM
  if (ntl_aligned(a, 16) && ntl_aligned(b, 16) && ntl_aligned(c, 16)) {
    const int64_t n4 = n / 4;
    const int tail = static_cast<int>(n % 4);
    int64_t blocks = (n4 + kThreads * kUnroll - 1) / (kThreads * kUnroll);
    if (blocks > max_blocks) blocks = max_blocks;
    if (blocks < 1) blocks = 1;
    ntl_launch_pdl(binary_f32_v4<OP>, dim3(static_cast<unsigned>(blocks)), dim3(kThreads), 0, stream,
                   reinterpret_cast<const float4*>(a), reinterpret_cast<const float4*>(b),
                   reinterpret_cast<float4*>(c), n4, a + n4 * 4, b + n4 * 4, c + n4 * 4, tail);
  } else {
    int64_t blocks = (n + kThreads - 1) / kThreads;
    if (blocks > max_blocks) blocks = max_blocks;
    ntl_launch_pdl(binary_f32_scalar<OP>, dim3(static_cast<unsigned>(blocks)), dim3(kThreads), 0, stream, a, b, c, n);
  }
  ntl_note_launch();
  return ntl_check_launch("elementwise launch");
}

}  // namespace

extern "C" int ntl_binary_f32(int op, const float* a, const float* b, float* c, int64_t n, ntl_stream_t stream) {
  NTL_REQUIRE(n >= 0, NTL_ERR_INVALID, "elementwise: n must be >= 0, got %lld", (long long)n);
  if (n == 0) return NTL_OK;
  NTL_REQUIRE(a && b && c, NTL_ERR_INVALID, "elementwise: NULL pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (op) {
    case 0: return launch_binary<0>(a, b, c, n, s);
    case 1: return launch_binary<1>(a, b, c, n, s);
    case 2: return launch_binary<2>(a, b, c, n, s);
    default: return ntl_fail(NTL_ERR_INVALID, "elementwise: unknown op %d", op);
  }
}

extern "C" int ntl_vadd_f32(const float* a, const float* b, float* c, int64_t n, ntl_stream_t stream) {
  return ntl_binary_f32(0, a, b, c, n, stream);
}
