// Shared helpers for the sm_100a kernels and their C-ABI wrappers.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "bfb_b200.h"

namespace bfb {

constexpr size_t kAlign = 256;

__host__ __device__ inline size_t align_up(size_t x, size_t a = kAlign) {
  return (x + a - 1) / a * a;
}

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Carves aligned sub-buffers out of one workspace.  With base == nullptr it
// only measures, so the size query and the real layout share one code path.
struct Carver {
  char* base;
  size_t off = 0;
  explicit Carver(void* b) : base(static_cast<char*>(b)) {}
  template <class T>
  T* take(size_t count) {
    size_t o = align_up(off);
    off = o + count * sizeof(T);
    return base ? reinterpret_cast<T*>(base + o) : nullptr;
  }
  size_t bytes() const { return align_up(off); }
};

// Debug builds (-DBFB_DEBUG_CHECKS, `python -m bevfusion_triton_b200._build
// --debug-checks`): device-side index checks count violations into a
// per-file error word instead of trapping; BFB_BAD(ok) is true (and counted)
// when `ok` fails, so the guarded access is skipped.  In release builds it
// is the constant false and compiles away.
#ifdef BFB_DEBUG_CHECKS
#define BFB_DEBUG_COUNTER() static __device__ unsigned long long bfb_violations_ = 0ull
#define BFB_BAD(ok) (!(ok) ? (atomicAdd(&bfb_violations_, 1ull), true) : false)
#define BFB_DEBUG_READER(fn)                                                               \
  int fn(uint64_t* v, int reset) {                                                         \
    unsigned long long x = 0ull;                                                           \
    BFB_CUDA(cudaMemcpyFromSymbol(&x, bfb_violations_, sizeof(x)));                        \
    if (reset) {                                                                           \
      const unsigned long long z = 0ull;                                                   \
      BFB_CUDA(cudaMemcpyToSymbol(bfb_violations_, &z, sizeof(z)));                        \
    }                                                                                      \
    *v += x;                                                                               \
    return BFB_OK;                                                                         \
  }
#else
#define BFB_DEBUG_COUNTER() static_assert(true, "")
#define BFB_BAD(ok) false
#define BFB_DEBUG_READER(fn) \
  int fn(uint64_t*, int) { return BFB_OK; }
#endif

// The error words of the kernel files (summed by bfb_debug_violations).
int debug_violations_bev(uint64_t* v, int reset);
int debug_violations_vox(uint64_t* v, int reset);
int debug_violations_scatter(uint64_t* v, int reset);
int debug_violations_spconv(uint64_t* v, int reset);
int debug_violations_spconv_conv(uint64_t* v, int reset);
int debug_violations_capi(uint64_t* v, int reset);

// A status armed by bfb_debug_inject_status for the next calls of the main
// entry points (host-side fault injection for tests), else BFB_OK.
int injected_status();
#define BFB_INJECT_POINT()                         \
  do {                                             \
    const int bfb_i_ = ::bfb::injected_status();   \
    if (bfb_i_ != BFB_OK) return bfb_i_;           \
  } while (0)

// Records the CUDA error text for bfb_last_cuda_error() and maps it to a status.
int record_cuda_error(cudaError_t e);
// Counts one kernel launch of this library (bfb_kernel_launches()).
void count_launch();

// Follows every kernel launch: counts it and maps a launch error to a status.
#define BFB_CHECK_LAUNCH()                                   \
  do {                                                       \
    ::bfb::count_launch();                                   \
    cudaError_t bfb_e_ = cudaGetLastError();                 \
    if (bfb_e_ != cudaSuccess) return ::bfb::record_cuda_error(bfb_e_); \
  } while (0)

#define BFB_CUDA(call)                                       \
  do {                                                       \
    cudaError_t bfb_e_ = (call);                             \
    if (bfb_e_ != cudaSuccess) return ::bfb::record_cuda_error(bfb_e_); \
  } while (0)

#define BFB_TRY(call)                 \
  do {                                \
    int bfb_s_ = (call);              \
    if (bfb_s_ != BFB_OK) return bfb_s_; \
  } while (0)

// fp32 <-> storage type conversions used by every kernel.
template <class T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <class T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

__device__ __forceinline__ unsigned lanemask_lt() {
  unsigned m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// Streaming (read-once) 16-byte load that does not allocate in L1.
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Streaming (write-once) 16-byte store, evict-first in L2.
__device__ __forceinline__ void st_stream16(void* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

// Division by a fixed 32-bit divisor with a multiply-high and shifts.
struct FastDiv {
  uint32_t d, magic, shift;
  FastDiv() = default;
  explicit FastDiv(uint32_t div) : d(div), magic(0), shift(0) {
    if (div > 1) {
      uint32_t s = 0;
      while ((1ull << s) < div) ++s;
      shift = s;
      magic = (uint32_t)((((1ull << 32) * ((1ull << s) - div)) / div) + 1);
    }
  }
  __device__ __forceinline__ uint32_t div(uint32_t n) const {
    if (d == 1) return n;
    const uint32_t t = __umulhi(n, magic);
    return (((n - t) >> 1) + t) >> (shift - 1);
  }
};

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline int dtype_size(int dt) {
  switch (dt) {
    case BFB_F32: return 4;
    case BFB_F16: return 2;
    case BFB_BF16: return 2;
    default: return 0;
  }
}

}  // namespace bfb
