// Library-wide C-ABI entry points: version, status text, last CUDA error.
#include <atomic>
#include <cstdio>
#include <cstring>

#include "common.cuh"

namespace bfb {
namespace {
thread_local char g_last_error[256] = "";
std::atomic<uint64_t> g_launches{0};
}

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int record_cuda_error(cudaError_t e) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s: %s", cudaGetErrorName(e), cudaGetErrorString(e));
  return BFB_ERR_CUDA;
}

}  // namespace bfb

extern "C" int bfb_abi_version(void) { return BFB_ABI_VERSION; }

extern "C" const char* bfb_status_string(int status) {
  switch (status) {
    case BFB_OK: return "ok";
    case BFB_ERR_INVALID_ARG: return "invalid argument";
    case BFB_ERR_UNSUPPORTED_DTYPE: return "unsupported dtype";
    case BFB_ERR_WORKSPACE: return "workspace missing or too small";
    case BFB_ERR_TOO_LARGE: return "sizes exceed the 32-bit index space";
    case BFB_ERR_CUDA: return "CUDA error";
    case BFB_ERR_DEVICE_STATUS: return "device-side check failed";
    case BFB_ERR_PLAN_MISMATCH: return "bev_pool plan was built for another geometry";
    default: return "unknown status";
  }
}

extern "C" const char* bfb_last_cuda_error(void) { return bfb::g_last_error; }

extern "C" uint64_t bfb_kernel_launches(void) { return bfb::g_launches.load(std::memory_order_relaxed); }
