/*
 * ntl_kernels.h — C ABI of libntl_kernels.so, the sm_100a kernel library behind the
 * ntilang-compatible Python surface.
 *
 * In the reference, every compiled kernel is reached through one boundary:
 * CompiledKernel.__call__ (python/ntilang/compiler.py:134-200) validates torch tensors and
 * calls `executable(*ffi_arguments)` (compiler.py:197), a TVM-FFI function that
 * `cute.compile(..., "--enable-tvm-ffi")` built from generated CuTe-DSL source
 * (python/ntilang/codegen.py:2206-2259).  Each entry point below replaces that FFI call
 * for one op family the reference's emitter produces; the Python side keeps the
 * reference's argument checks and passes raw device pointers, sizes and the caller's
 * CUDA stream (torch's current stream, which is what TVM-FFI's environment stream
 * follows in the reference — pinned by tests/test_gpu.py:90-101).
 *
 * Conventions
 *  - All pointers are device pointers owned by the caller; tensors are dense row-major.
 *  - fp16 data is passed as `const uint16_t*` (IEEE binary16 bit patterns).
 *  - `stream` is a cudaStream_t (NULL = legacy default stream).  Launches are
 *    asynchronous; nothing here synchronises the stream or allocates device memory.
 *  - Return 0 on success or an NTL_ERR_* code; ntl_last_error() then describes the
 *    failure (thread-local).  Argument errors are detected on the host before launch.
 */
#ifndef NTL_KERNELS_H
#define NTL_KERNELS_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* ntl_stream_t;

enum {
  NTL_OK = 0,
  NTL_ERR_INVALID = 1,     /* bad size / null pointer / unsupported parameter */
  NTL_ERR_UNSUPPORTED = 2, /* shape outside what the kernels implement */
  NTL_ERR_CUDA = 3,        /* a CUDA runtime call or launch failed */
  NTL_ERR_TIMEOUT = 4,     /* a bounded device-side wait gave up (see ntl_device_status) */
  NTL_ERR_ALIGNMENT = 5    /* pointer alignment not met for the requested path */
};

/* Library version (major*10000 + minor*100 + patch). */
int ntl_version(void);

/* Message for the last non-zero return on this thread ("" if none). */
const char* ntl_last_error(void);

/* Vector add C[i] = A[i] + B[i] for i < n (fp32).  Replaces the FFI call of the
 * elementwise kernel emitted for examples/vector_add.py:5-10 (codegen.py:1494-1517 store,
 * :1694-1734 parallel loop).  Bit-exact: one IEEE fp32 add per element. */
int ntl_vadd_f32(const float* a, const float* b, float* c, int64_t n, ntl_stream_t stream);

/* Elementwise binary op over n fp32 elements: op 0 = add, 1 = sub, 2 = mul.  Same
 * reference emitter as ntl_vadd_f32 (codegen.py:1494-1517, :1694-1734). */
int ntl_binary_f32(int op, const float* a, const float* b, float* c, int64_t n, ntl_stream_t stream);

/* Inclusive prefix sum along each row of a [rows, cols] fp32 matrix; reverse != 0 scans
 * from the last column.  Replaces the FFI call of the warp scan emitted by
 * python/ntilang/scan.py:132-240 for examples/cumsum.py:7-14.  The addition DAG is the
 * reference's: 32-column Hillis-Steele segments (offsets 1,2,4,8,16) followed by a
 * sequential carry carry_{s+1} = seg_s[last] + carry_s starting from +0
 * (scan.py:168-237, evaluate :349-389), so results are bit-identical to it. */
int ntl_cumsum_f32(const float* x, float* y, int64_t rows, int64_t cols, int reverse, ntl_stream_t stream);

/* Inclusive prefix maximum along each row (T.cummax), same layout and reverse flag as
 * ntl_cumsum_f32.  Replaces the FFI call of the scan emitted for T.cummax
 * (python/ntilang/scan.py:83-115, examples/scan.py:7-21): identity -inf, combine fmax
 * (a NaN operand is ignored, +0 orders above -0; scan.py:26-29, :366-374). */
int ntl_cummax_f32(const float* x, float* y, int64_t rows, int64_t cols, int reverse, ntl_stream_t stream);

/* Row softmax y = exp(x - max) / sum(exp(x - max)) over [rows, cols] fp32.  Replaces the
 * FFI call of the row-reduction kernel emitted for examples/softmax.py:9-25
 * (codegen.py:1028-1240).  Sums follow the reference's balanced tree over the row padded
 * to the next power of two (codegen.py:1094-1151). */
int ntl_softmax_f32(const float* x, float* y, int64_t rows, int64_t cols, ntl_stream_t stream);

/* RMSNorm y = (x * rsqrt(sum(x^2) * inv_n + eps)) * w over [rows, cols] fp32, w[cols].
 * Replaces the FFI call of the kernel emitted for examples/rmsnorm.py:13-37; inv_n is the
 * program's constant (the reference multiplies by 1/n, rmsnorm.py:10,34). */
int ntl_rmsnorm_f32(const float* x, const float* w, float* y, int64_t rows, int64_t cols, float eps,
                    float inv_n, ntl_stream_t stream);

/* LayerNorm y = ((x - mean) * rstd) * w + b over [rows, cols] fp32, w[cols], b[cols], with
 * mean = sum(x) * inv_n and rstd = rsqrt(sum((x - mean)^2) * inv_n + eps), both sums the
 * reference's balanced tree over the row padded to the next power of two.  Replaces the FFI
 * call of the kernel emitted for examples/layernorm.py:18-43 (inv_n = 1/n at :10). */
int ntl_layernorm_f32(const float* x, const float* w, const float* b, float* y, int64_t rows, int64_t cols,
                      float eps, float inv_n, ntl_stream_t stream);

/* b[n, m] = a[m, n]^T, fp32 row-major, out of place (bit-exact copy).  Replaces the FFI call
 * of the shared-memory transpose emitted for examples/transpose.py:5-15. */
int ntl_transpose_f32(const float* a, float* b, int64_t m, int64_t n, ntl_stream_t stream);

/* Bias modes of ntl_gemm_f16_f32. */
enum { NTL_BIAS_NONE = 0, NTL_BIAS_N = 1, NTL_BIAS_MN = 2, NTL_BIAS_M = 3 };

/* C[M,N] (fp32) = epilogue(A[M,K] @ B), fp16 operands, fp32 accumulation.
 *   B is [K,N] row-major (b_trans = 0) or [N,K] row-major (b_trans = 1, T.gemm transpose_B).
 *   epilogue: v = alpha * acc (+ bias[n] | bias[m,n] | bias[m]); if relu: v = max(v, 0).
 * Replaces the FFI call of the GEMM emitted by codegen.py:969-1026 + :1611-1693 for
 * examples/matmul.py:17-29 and its fused epilogue (codegen.py:1694-1734,
 * examples/matmul_relu.py:31-38).  Aligned shapes (K, N multiples of 8; 16-byte aligned
 * pointers) run the tcgen05/TMEM kernel; other shapes run a CUDA-core tiled kernel. */
int ntl_gemm_f16_f32(const uint16_t* a, const uint16_t* b, float* c, const float* bias, int bias_mode,
                     float alpha, int relu, int64_t M, int64_t N, int64_t K, int b_trans, ntl_stream_t stream);

/* Workspace (bytes) ntl_gemm_f16_f32_ws needs for this shape on the current device; 0 when
 * every output tile is computed data-parallel.  Same reference counterpart as
 * ntl_gemm_f16_f32 (the workspace replaces nothing in the reference: its GEMM has no
 * cross-CTA reduction). */
int ntl_gemm_workspace_size(int64_t M, int64_t N, int64_t K, int b_trans, uint64_t* bytes_out);

/* ntl_gemm_f16_f32 with a caller-owned workspace of at least ntl_gemm_workspace_size bytes
 * (16-byte aligned).  Its first 4 KB hold flag words that must be zero before the first use;
 * every successful call leaves them zero again, whatever the shape, so one workspace serves
 * every shape that fits it.  The last, partial wave of output tiles is split along K and
 * reduced through the workspace: over all SMs (stream-K) for M <= 128, into 2-4 pieces on
 * idle CTA pairs for M > 128.  Calls sharing a workspace must not overlap on the GPU.
 * Replaces the same FFI call as ntl_gemm_f16_f32 (codegen.py:969-1026). */
int ntl_gemm_f16_f32_ws(const uint16_t* a, const uint16_t* b, float* c, const float* bias, int bias_mode,
                        float alpha, int relu, int64_t M, int64_t N, int64_t K, int b_trans, void* workspace,
                        uint64_t workspace_bytes, ntl_stream_t stream);

/* ntl_gemm_f16_f32_ws for callers that cannot allocate device memory (e.g. a plugin host
 * that passes only tensors and a stream, or a runtime with the device allocator switched
 * off): the split-K scratch lives in a 16 MiB file-scope device array that every GPU
 * loading the library holds until exit.  Shapes whose plan needs more scratch than that
 * return NTL_ERR_UNSUPPORTED; the need is decided as in ntl_gemm_f16_f32_ws, so operands the
 * TMA path cannot address (A or B not 16-byte aligned, K or N not a multiple of 8) take the
 * CUDA-core path, use no scratch and are never refused for size.  The first call on a device
 * (and the first after a cudaDeviceReset there) looks up the array's device address
 * (cudaGetSymbolAddress) and should come before any stream capture.  Calls share the array:
 * a call that uses it first enqueues a 4 KB cudaMemsetAsync of the flag words on the
 * caller's stream, then the kernel; calls that overlap on the GPU race.  No counterpart in
 * the reference (its kernels take no scratch). */
int ntl_gemm_f16_f32_noalloc(const uint16_t* a, const uint16_t* b, float* c, const float* bias, int bias_mode,
                             float alpha, int relu, int64_t M, int64_t N, int64_t K, int b_trans,
                             ntl_stream_t stream);

/* FlashAttention-2 forward, fp16 Q,K,V,O [batch, heads, seq, dim] row-major.
 *   O = softmax_base2((Q K^T) * scale_log2 [causal: key <= query]) V, with P rounded to fp16
 *   before the P V product and fp32 softmax statistics.
 * Non-causal launches one CTA per (batch, head, 256-query block).  Causal does the same unless
 * the blocks, paired heaviest with lightest, fill at least 95% of whole rounds of one CTA per
 * SM: then it launches that persistent grid, which runs the pairs in a fixed order, so kernels
 * on other streams share SMs with it only as its CTAs finish.  Both grids give bit-identical
 * results; ntl_fa2_set_causal_grid overrides the choice.
 * Replaces the FFI call of the kernel emitted for examples/flash_attention.py:26-79
 * (scale = log2(e)/sqrt(d) at :23, causal fill at :56-62, P cast at :74-75). */
int ntl_fa2_fwd_f16(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* o, int64_t batch,
                    int64_t heads, int64_t seq, int64_t dim, float scale_log2, int causal, ntl_stream_t stream);

/* Grid of the causal ntl_fa2_fwd_f16 calls this process makes from now on: NTL_FA2_GRID_AUTO
 * (the rule above, the default), NTL_FA2_GRID_PERSISTENT or NTL_FA2_GRID_PER_BLOCK.
 * Process-wide, like ntl_set_wait_limit; NTL_ERR_INVALID for any other value.  No reference
 * counterpart. */
#define NTL_FA2_GRID_AUTO 0
#define NTL_FA2_GRID_PERSISTENT 1
#define NTL_FA2_GRID_PER_BLOCK 2
int ntl_fa2_set_causal_grid(int mode);

/* Generic elementwise programs (outside the families above): run-time compiled kernels.
 * ntl_rtc_build compiles CUDA C `source` (one extern "C" __global__ function named
 * `kernel_name`) with NVRTC for sm_100a on the host, no GPU needed, and returns a handle;
 * ntl_rtc_launch runs it as a 1-D grid of grid_x blocks of block_x threads on `stream`, with
 * `args` the kernel's argument pointers in cuLaunchKernel form.  Together they replace the
 * reference's CompiledKernel.build() / executable(*ffi_arguments) pair for such programs
 * (python/ntilang/compiler.py:51-71, :197).  A compile error returns NTL_ERR_INVALID with the
 * NVRTC log in ntl_last_error(). */
int ntl_rtc_build(const char* source, const char* kernel_name, uint64_t* handle_out);
int ntl_rtc_launch(uint64_t handle, uint64_t grid_x, uint32_t block_x, void** args, ntl_stream_t stream);

/* Device status word of the bounded waits in the tcgen05 kernels on the current device:
 * 0 = no timeout since the last clear, else a code naming the wait that gave up.  Reading
 * it synchronises the device.  No reference counterpart (its kernels have no bounded
 * waits); exposed so callers can turn a timed-out launch into an error. */
int ntl_device_status(uint32_t* status_out);
int ntl_clear_device_status(void);

/* Spin limit of every bounded wait (default 1<<26 polls).  Test hook: a limit of 1 makes
 * waits give up early so the timeout path can be exercised without hanging anything.
 * No reference counterpart. */
int ntl_set_wait_limit(int64_t polls);

/* Number of kernel launches issued by this library in this process (all devices). */
int64_t ntl_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* NTL_KERNELS_H */
