// Library-level entry points: version, status strings, last-error detail,
// and the host helpers shared by the kernel files.
#include <atomic>
#include <mutex>
#include <string>

#include "common.cuh"

namespace pkm {

static thread_local std::string g_last_error;

void set_last_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
  set_last_error(msg);
  return code;
}

int check_cuda(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return PKM_OK;
  set_last_error(std::string(what) + ": " + cudaGetErrorString(e));
  return PKM_ERR_CUDA;
}

// SM count of the current device, cached per device ordinal; host threads
// may call into the library at the same time, so the entries are atomics
// (two threads that miss together both store the same value).
int num_sms() {
  static std::atomic<int> cache[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  int v = cache[dev].load(std::memory_order_relaxed);
  if (v == 0) {
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    v = v > 0 ? v : 1;
    cache[dev].store(v, std::memory_order_relaxed);
  }
  return v;
}

}  // namespace pkm

extern "C" int pkm_version(void) { return 100; }

extern "C" const char* pkm_status_string(int status) {
  switch (status) {
    case PKM_OK:
      return "ok";
    case PKM_ERR_INVALID_ARG:
      return "invalid argument";
    case PKM_ERR_UNSUPPORTED:
      return "unsupported size";
    case PKM_ERR_CUDA:
      return "CUDA error";
    case PKM_ERR_WORKSPACE:
      return "workspace too small";
    default:
      return "unknown status";
  }
}

extern "C" const char* pkm_last_error(void) { return pkm::g_last_error.c_str(); }
