// Library-level entry points: status strings, error bookkeeping, device cache.
#include "common.cuh"

namespace iron {

static thread_local int g_last_cuda_error = 0;

void set_last_cuda_error(cudaError_t e) { g_last_cuda_error = static_cast<int>(e); }

int sm_count() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

}  // namespace iron

extern "C" const char *iron_strerror(int status) {
  switch (status) {
    case IRON_OK: return "ok";
    case IRON_ERR_NULL: return "a required pointer is NULL";
    case IRON_ERR_SHAPE: return "invalid or inconsistent shape";
    case IRON_ERR_ALIGN: return "pointer or leading dimension not 16-byte aligned";
    case IRON_ERR_UNSUPPORTED: return "configuration not supported by this build";
    case IRON_ERR_CUDA: return "CUDA runtime error (see iron_last_cuda_error)";
    case IRON_ERR_WORKSPACE: return "workspace too small";
    case IRON_ERR_TIMEOUT: return "bounded device-side wait timed out";
    case IRON_ERR_ARG: return "invalid argument";
    default: return "unknown status";
  }
}

extern "C" int iron_last_cuda_error(void) { return iron::g_last_cuda_error; }

extern "C" int iron_abi_version(void) { return (1 << 16) | 1; }
