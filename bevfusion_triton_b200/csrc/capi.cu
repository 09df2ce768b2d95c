// Library-wide C-ABI entry points: version, status text, last CUDA error.
#include <atomic>
#include <cstdio>
#include <cstring>

#include "common.cuh"

namespace bfb {

BFB_DEBUG_COUNTER();
BFB_DEBUG_READER(debug_violations_capi)

namespace {
thread_local char g_last_error[256] = "";
std::atomic<uint64_t> g_launches{0};
std::atomic<int> g_inject_status{0};
std::atomic<int64_t> g_inject_calls{0};

// Counts `k` synthetic violations (tests the error word of a debug build).
__global__ void debug_selftest_kernel(int k) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < k && BFB_BAD(i < 0)) return;
}
}

int injected_status() {
  if (g_inject_calls.load(std::memory_order_relaxed) <= 0) return BFB_OK;
  if (g_inject_calls.fetch_sub(1) <= 0) return BFB_OK;
  return g_inject_status.load();
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

extern "C" int bfb_debug_checks_enabled(void) {
#ifdef BFB_DEBUG_CHECKS
  return 1;
#else
  return 0;
#endif
}

extern "C" int bfb_debug_violations(uint64_t* count, int reset) {
  if (!count) return BFB_ERR_INVALID_ARG;
  *count = 0;
  BFB_TRY(bfb::debug_violations_bev(count, reset));
  BFB_TRY(bfb::debug_violations_vox(count, reset));
  BFB_TRY(bfb::debug_violations_scatter(count, reset));
  BFB_TRY(bfb::debug_violations_spconv(count, reset));
  BFB_TRY(bfb::debug_violations_spconv_conv(count, reset));
  BFB_TRY(bfb::debug_violations_capi(count, reset));
  return BFB_OK;
}

extern "C" int bfb_debug_selftest(int k, void* stream) {
  if (k < 0) return BFB_ERR_INVALID_ARG;
  if (k == 0) return BFB_OK;
  bfb::debug_selftest_kernel<<<(k + 255) / 256, 256, 0, bfb::as_stream(stream)>>>(k);
  BFB_CHECK_LAUNCH();
  return BFB_OK;
}

extern "C" int bfb_debug_inject_status(int status, int calls) {
  if (calls < 0 || status > 0) return BFB_ERR_INVALID_ARG;
  bfb::g_inject_status.store(status);
  bfb::g_inject_calls.store(status == BFB_OK ? 0 : calls);
  return BFB_OK;
}
