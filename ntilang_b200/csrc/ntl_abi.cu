// Library-wide host state of libntl_kernels.so: error messages, launch counter, the
// bounded-wait limit and the device status readers.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>

#include "ntl_common.cuh"

namespace {
thread_local std::string g_last_error;
std::atomic<int64_t> g_launches{0};
std::atomic<int64_t> g_wait_limit{int64_t(1) << 26};
constexpr int kMaxDevices = 64;
std::atomic<int> g_sms[kMaxDevices];
}  // namespace

int ntl_fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int ntl_check_launch(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return ntl_fail(NTL_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
  return NTL_OK;
}

void ntl_note_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

int64_t ntl_wait_limit() { return g_wait_limit.load(std::memory_order_relaxed); }

int ntl_num_sms(int* sms_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return ntl_fail(NTL_ERR_CUDA, "cudaGetDevice failed");
  if (dev >= 0 && dev < kMaxDevices) {
    int cached = g_sms[dev].load(std::memory_order_relaxed);
    if (cached > 0) {
      *sms_out = cached;
      return NTL_OK;
    }
  }
  int sms = 0;
  cudaError_t err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (err != cudaSuccess) return ntl_fail(NTL_ERR_CUDA, "cudaDeviceGetAttribute: %s", cudaGetErrorString(err));
  if (dev >= 0 && dev < kMaxDevices) g_sms[dev].store(sms, std::memory_order_relaxed);
  *sms_out = sms;
  return NTL_OK;
}

extern "C" {

int ntl_version(void) { return 100; }

const char* ntl_last_error(void) { return g_last_error.c_str(); }

int64_t ntl_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int ntl_set_wait_limit(int64_t polls) {
  if (polls < 1) return ntl_fail(NTL_ERR_INVALID, "wait limit must be >= 1, got %lld", (long long)polls);
  g_wait_limit.store(polls, std::memory_order_relaxed);
  return NTL_OK;
}

int ntl_device_status(uint32_t* status_out) {
  if (status_out == nullptr) return ntl_fail(NTL_ERR_INVALID, "status_out is NULL");
  uint32_t s = ntl_gemm_status_read(0);
  if (s == 0) s = ntl_fa2_status_read(0);
  *status_out = s;
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return ntl_fail(NTL_ERR_CUDA, "reading device status: %s", cudaGetErrorString(err));
  return NTL_OK;
}

int ntl_clear_device_status(void) {
  ntl_gemm_status_read(1);
  ntl_fa2_status_read(1);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return ntl_fail(NTL_ERR_CUDA, "clearing device status: %s", cudaGetErrorString(err));
  return NTL_OK;
}

}  // extern "C"
