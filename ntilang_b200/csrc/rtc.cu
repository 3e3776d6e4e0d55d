// Run-time compiled kernels: CUDA C source -> NVRTC -> sm_100a cubin -> module per device.
//
// This is the back end of the generic elementwise path (programs outside the recognised op
// families): ntilang_b200.pointwise writes one CUDA C kernel per program and the reference's
// `CompiledKernel.build()` / `executable(*args)` pair (python/ntilang/compiler.py:51-71,
// :197) becomes ntl_rtc_build() + ntl_rtc_launch() here.
//
// * ntl_rtc_build compiles on the host only (NVRTC needs no GPU): options
//   --gpu-architecture=sm_100a, --fmad=false (every multiply and add rounds separately, as the
//   reference's evaluator computes), IEEE division and square root.  Cubins are cached in
//   memory by source text and on disk under $NTL_RTC_CACHE (default
//   ~/.cache/ntilang_b200/rtc) by a 128-bit hash of compiler version + options + source.
// * ntl_rtc_launch loads the cubin into the current device's primary context on first use
//   (cuModuleLoadData through the runtime's driver entry points) and launches a 1-D grid with
//   cuLaunchKernel on the caller's stream.
// NVRTC is opened with dlopen on first use, so the library itself loads without it.
#include <dlfcn.h>
#include <nvrtc.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "ntl_common.cuh"

namespace {

struct Nvrtc {
  decltype(&nvrtcCreateProgram) create = nullptr;
  decltype(&nvrtcCompileProgram) compile = nullptr;
  decltype(&nvrtcGetProgramLogSize) log_size = nullptr;
  decltype(&nvrtcGetProgramLog) log = nullptr;
  decltype(&nvrtcGetCUBINSize) cubin_size = nullptr;
  decltype(&nvrtcGetCUBIN) cubin = nullptr;
  decltype(&nvrtcDestroyProgram) destroy = nullptr;
  decltype(&nvrtcGetErrorString) error = nullptr;
  decltype(&nvrtcVersion) version = nullptr;
  bool ok = false;
  std::string why;
};

const Nvrtc& nvrtc() {
  static Nvrtc api;
  static std::once_flag once;
  std::call_once(once, [] {
    const char* env = std::getenv("NTL_NVRTC_LIB");
    const char* names[] = {env, "libnvrtc.so.12", "libnvrtc.so", "/usr/local/cuda/lib64/libnvrtc.so.12"};
    void* h = nullptr;
    for (const char* n : names)
      if (n != nullptr && (h = dlopen(n, RTLD_NOW | RTLD_LOCAL)) != nullptr) break;
    if (h == nullptr) {
      api.why = "libnvrtc.so.12 not found (set NTL_NVRTC_LIB)";
      return;
    }
#define NTL_SYM(field, name)                                                   \
  api.field = reinterpret_cast<decltype(api.field)>(dlsym(h, name));           \
  if (api.field == nullptr) {                                                  \
    api.why = std::string("NVRTC lacks ") + name;                              \
    return;                                                                    \
  }
    NTL_SYM(create, "nvrtcCreateProgram");
    NTL_SYM(compile, "nvrtcCompileProgram");
    NTL_SYM(log_size, "nvrtcGetProgramLogSize");
    NTL_SYM(log, "nvrtcGetProgramLog");
    NTL_SYM(cubin_size, "nvrtcGetCUBINSize");
    NTL_SYM(cubin, "nvrtcGetCUBIN");
    NTL_SYM(destroy, "nvrtcDestroyProgram");
    NTL_SYM(error, "nvrtcGetErrorString");
    NTL_SYM(version, "nvrtcVersion");
#undef NTL_SYM
    api.ok = true;
  });
  return api;
}

// Driver entry points reached through the runtime (no link-time dependency on libcuda).
struct Driver {
  CUresult (*load)(CUmodule*, const void*) = nullptr;
  CUresult (*get_function)(CUfunction*, CUmodule, const char*) = nullptr;
  CUresult (*launch)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, CUstream,
                     void**, void**) = nullptr;
  bool ok = false;
};

const Driver& driver() {
  static Driver d;
  static std::once_flag once;
  std::call_once(once, [] {
    auto get = [](const char* name) -> void* {
      void* p = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
        return nullptr;
      return p;
    };
    d.load = reinterpret_cast<decltype(d.load)>(get("cuModuleLoadData"));
    d.get_function = reinterpret_cast<decltype(d.get_function)>(get("cuModuleGetFunction"));
    d.launch = reinterpret_cast<decltype(d.launch)>(get("cuLaunchKernel"));
    d.ok = d.load && d.get_function && d.launch;
  });
  return d;
}

constexpr int kMaxDevices = 64;

struct RtcKernel {
  std::string name;
  std::vector<char> cubin;
  CUfunction fn[kMaxDevices] = {};
  std::mutex mu;
};

std::mutex g_mu;
std::vector<std::unique_ptr<RtcKernel>> g_kernels;  // handle = index + 1
std::unordered_map<std::string, uint64_t> g_by_source;

const char* const kOptions[] = {"--gpu-architecture=sm_100a", "--fmad=false", "--prec-div=true",
                                "--prec-sqrt=true", "--ftz=false", "-std=c++17", "-default-device"};

uint64_t fnv1a(const std::string& s, uint64_t h) {
  for (unsigned char c : s) {
    h ^= c;
    h *= 1099511628211ull;
  }
  return h;
}

std::string cache_path(const std::string& key) {
  std::string dir;
  if (const char* d = std::getenv("NTL_RTC_CACHE")) {
    dir = d;
  } else if (const char* home = std::getenv("HOME")) {
    dir = std::string(home) + "/.cache/ntilang_b200/rtc";
  } else {
    return "";
  }
  if (dir == "off") return "";
  // mkdir -p
  for (size_t i = 1; i <= dir.size(); ++i)
    if (i == dir.size() || dir[i] == '/') mkdir(dir.substr(0, i).c_str(), 0755);
  char name[64];
  snprintf(name, sizeof(name), "/%016llx%016llx.cubin", (unsigned long long)fnv1a(key, 14695981039346656037ull),
           (unsigned long long)fnv1a(key, 1469598103934665603ull ^ 0x9e3779b97f4a7c15ull));
  return dir + name;
}

bool read_file(const std::string& path, std::vector<char>* out) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (f == nullptr) return false;
  std::vector<char> buf;
  char tmp[65536];
  size_t n;
  while ((n = std::fread(tmp, 1, sizeof(tmp), f)) > 0) buf.insert(buf.end(), tmp, tmp + n);
  std::fclose(f);
  if (buf.empty()) return false;
  out->swap(buf);
  return true;
}

void write_file(const std::string& path, const std::vector<char>& data) {
  const std::string tmp = path + ".tmp" + std::to_string(static_cast<long long>(getpid()));
  FILE* f = std::fopen(tmp.c_str(), "wb");
  if (f == nullptr) return;
  const bool ok = std::fwrite(data.data(), 1, data.size(), f) == data.size();
  std::fclose(f);
  if (ok) std::rename(tmp.c_str(), path.c_str());
  else std::remove(tmp.c_str());
}

int compile_cubin(const std::string& source, const std::string& name, std::vector<char>* cubin) {
  const Nvrtc& api = nvrtc();
  if (!api.ok) return ntl_fail(NTL_ERR_UNSUPPORTED, "run-time compilation unavailable: %s", api.why.c_str());
  int major = 0, minor = 0;
  api.version(&major, &minor);
  std::string key = std::to_string(major) + "." + std::to_string(minor);
  for (const char* o : kOptions) key += std::string("\n") + o;
  key += "\n" + name + "\n" + source;
  const std::string path = cache_path(key);
  if (!path.empty() && read_file(path, cubin)) return NTL_OK;

  nvrtcProgram prog;
  nvrtcResult r = api.create(&prog, source.c_str(), (name + ".cu").c_str(), 0, nullptr, nullptr);
  if (r != NVRTC_SUCCESS) return ntl_fail(NTL_ERR_CUDA, "nvrtcCreateProgram: %s", api.error(r));
  r = api.compile(prog, static_cast<int>(sizeof(kOptions) / sizeof(kOptions[0])), kOptions);
  if (r != NVRTC_SUCCESS) {
    size_t n = 0;
    api.log_size(prog, &n);
    std::string log(n, '\0');
    if (n > 0) api.log(prog, &log[0]);
    api.destroy(&prog);
    return ntl_fail(NTL_ERR_INVALID, "NVRTC could not compile %s: %s", name.c_str(), log.c_str());
  }
  size_t n = 0;
  api.cubin_size(prog, &n);
  cubin->resize(n);
  api.cubin(prog, cubin->data());
  api.destroy(&prog);
  if (!path.empty()) write_file(path, *cubin);
  return NTL_OK;
}

RtcKernel* kernel_of(uint64_t handle) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (handle == 0 || handle > g_kernels.size()) return nullptr;
  return g_kernels[handle - 1].get();
}

}  // namespace

extern "C" int ntl_rtc_build(const char* source, const char* kernel_name, uint64_t* handle_out) {
  NTL_REQUIRE(source && kernel_name && handle_out, NTL_ERR_INVALID, "rtc_build: NULL argument");
  const std::string src(source), name(kernel_name);
  const std::string key = name + '\0' + src;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_by_source.find(key);
    if (it != g_by_source.end()) {
      *handle_out = it->second;
      return NTL_OK;
    }
  }
  auto k = std::make_unique<RtcKernel>();
  k->name = name;
  if (int rc = compile_cubin(src, name, &k->cubin)) return rc;
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_by_source.find(key);
  if (it != g_by_source.end()) {
    *handle_out = it->second;
    return NTL_OK;
  }
  g_kernels.push_back(std::move(k));
  const uint64_t h = g_kernels.size();
  g_by_source.emplace(key, h);
  *handle_out = h;
  return NTL_OK;
}

extern "C" int ntl_rtc_launch(uint64_t handle, uint64_t grid_x, uint32_t block_x, void** args,
                              ntl_stream_t stream) {
  RtcKernel* k = kernel_of(handle);
  NTL_REQUIRE(k != nullptr, NTL_ERR_INVALID, "rtc_launch: unknown kernel handle %llu", (unsigned long long)handle);
  if (grid_x == 0) return NTL_OK;
  NTL_REQUIRE(grid_x <= 0x7fffffffull, NTL_ERR_UNSUPPORTED, "rtc_launch: grid of %llu blocks is too large",
              (unsigned long long)grid_x);
  NTL_REQUIRE(block_x >= 1 && block_x <= 1024, NTL_ERR_INVALID, "rtc_launch: block of %u threads", block_x);
  const Driver& drv = driver();
  NTL_REQUIRE(drv.ok, NTL_ERR_CUDA, "rtc_launch: CUDA driver entry points unavailable");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return ntl_fail(NTL_ERR_CUDA, "cudaGetDevice failed");
  NTL_REQUIRE(dev >= 0 && dev < kMaxDevices, NTL_ERR_UNSUPPORTED, "rtc_launch: device %d", dev);
  CUfunction fn;
  {
    std::lock_guard<std::mutex> lk(k->mu);
    if (k->fn[dev] == nullptr) {
      // cudaFree(nullptr) makes the device's primary context current on this thread.
      if (cudaFree(nullptr) != cudaSuccess) return ntl_fail(NTL_ERR_CUDA, "rtc_launch: no CUDA context");
      CUmodule mod;
      CUresult r = drv.load(&mod, k->cubin.data());
      if (r != CUDA_SUCCESS) return ntl_fail(NTL_ERR_CUDA, "cuModuleLoadData(%s) failed (%d)", k->name.c_str(), int(r));
      r = drv.get_function(&k->fn[dev], mod, k->name.c_str());
      if (r != CUDA_SUCCESS)
        return ntl_fail(NTL_ERR_CUDA, "cuModuleGetFunction(%s) failed (%d)", k->name.c_str(), int(r));
    }
    fn = k->fn[dev];
  }
  CUresult r = drv.launch(fn, static_cast<unsigned>(grid_x), 1, 1, block_x, 1, 1, 0, static_cast<CUstream>(stream),
                          args, nullptr);
  if (r != CUDA_SUCCESS) return ntl_fail(NTL_ERR_CUDA, "cuLaunchKernel(%s) failed (%d)", k->name.c_str(), int(r));
  ntl_note_launch();
  return NTL_OK;
}
