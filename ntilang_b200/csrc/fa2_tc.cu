// FlashAttention-2 forward on sm_100a (tcgen05 + TMEM).  Bring-up placeholder: the
// entry point validates its arguments and reports the op as not yet available.
#include "ntl_common.cuh"

namespace {
__device__ uint32_t g_fa2_status;
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
  (void)q, (void)k, (void)v, (void)o, (void)batch, (void)heads, (void)seq, (void)dim, (void)scale_log2,
      (void)causal, (void)stream;
  return ntl_fail(NTL_ERR_UNSUPPORTED, "fa2: kernel not built yet");
}
