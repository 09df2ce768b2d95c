// Sparse convolution and sparse max-pooling over a rulebook, for sm_100a.
//
// Reference semantics: ops/spconv/src/spconv_triton.py
//   :981-1007  indice_conv: out = zeros[num_out, Cout]; for every rule k with
//              pairs, out[out_idx] += features[in_idx] @ filters[k]
//              (filters viewed [K, Cin, Cout]); `inverse` swaps the pair slots
//   :1010-1032 fused_indice_conv: + bias unless subm
//   :1035-1061 indice_conv_backward: input_grad[in_idx] += out_bp[out_idx] @
//              filters[k]^T, filters_grad[k] = features[in_idx]^T @ out_bp[out_idx]
//   :1064-1082 indice_maxpool: out = zeros; out[out_idx] = amax(out, features[in_idx])
//              (so a pooled value is never below 0)
//   :1085-1111 indice_maxpool_backward: input_grad[in_idx] += out_bp[out_idx]
//              where features[in_idx] == out_features[out_idx]
//
// Design.  The tensor-core path is output-stationary: the rulebook
// (rule-major pairs) is turned into a neighbour table nbr[row][k] (the input
// feeding output `row` through offset k, or -1) by one scatter kernel, and
// every output row is produced by ONE thread block as a sum over k, written
// once.  The FMA path (fp32 and other widths) is rule-major: the offsets run
// in ascending order, each reusing its filter over 64 pairs at a time, and
// add into the output rows.  Neither uses atomics; both are deterministic.
// The backward's input gradient is the same operation with the pair slots
// swapped and the filters transposed, so it runs through the same kernels.
//
//   spc_nbr_kernel         rulebook -> nbr_out[n_out][K] (+ nbr_in[n_in][K])
//   spc_conv_tc_kernel     fp16 / bf16, channels multiples of 16: a tile of
//                          128 output rows is one tcgen05 GEMM chain
//                          (M = 128, N = out channels, K = in channels per
//                          offset) with the fp32 accumulator in tensor memory.
//                          The gathered rows are staged by cp.async (zero-filled
//                          for missing neighbours) in the K-major core-matrix
//                          layout; the offset's filter block, laid out in that
//                          layout once per call by spc_prep_tc_kernel, arrives
//                          by one cp.async.bulk copy completing on an mbarrier.
//                          Two stages: the next offset's rows load while the
//                          tensor cores work on the current one.
//   spc_rule_kernel        every other case (fp32, odd channel counts): one
//                          launch per offset in ascending order, 64 of the
//                          rule's pairs per block, the filter in shared memory,
//                          fp32 FMA, read-modify-write of the output rows
//   spc_dw_plan_kernel +   filters_grad: every rule's pairs cut into chunks of
//   spc_dw_tc_kernel /     one common length (planned on the device from the
//   spc_dw_kernel +        rule counts), a fp32 partial per chunk (tcgen05 for
//   spc_dw_reduce_kernel   fp16 / bf16, reduction over pairs; else fp32 FMA),
//                          summed per rule in a fixed two-level order
//   spc_maxpool_kernel / spc_maxpool_bwd_kernel
//
// Every wait on an mbarrier is bounded; a wait that gives up counts into a
// device error word (bfb_spconv_timeouts) and the block still waits, bounded,
// for its own tensor-core work before it frees its tensor memory and returns.
#include <algorithm>
#include <cstdlib>
#include <type_traits>

#include "common.cuh"

namespace bfb {

BFB_DEBUG_COUNTER();
BFB_DEBUG_READER(debug_violations_spconv_conv)

namespace {

__device__ unsigned long long g_spc_timeouts = 0ull;

constexpr int kTcRows = 128;          // output rows per tensor-core tile (UMMA M)
constexpr int kTcThreads = 128;       // one thread per tile row in the epilogue
constexpr int kSimtThreads = 256;     // 16 x 16 threads, 4 x 4 outputs each
constexpr int kSimtChunk = 32;        // input channels staged per step
constexpr int kMaxK = 343;            // kernel volume up to 7x7x7
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s: a correct wait takes microseconds

// ------------------------------------------------------------------ helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait for the phase of parity `parity` to complete, polling (non-blocking
// test_wait) for at most kWaitNs of wall time; false if it gave up.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0;; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
    if ((i & 255u) == 255u && globaltimer_ns() - t0 > kWaitNs) break;
  }
  atomicAdd(&g_spc_timeouts, 1ull);
  return false;
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Plain (non-multicast) bulk copy global -> this CTA's shared memory.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor, K-major, no swizzle: core matrices of 8
// rows x 16 bytes stored as contiguous 128-byte blocks; `lbo` = bytes between
// the two core matrices of one K=16 step, `sbo` = bytes between 8-row groups.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3fff);
  d |= (uint64_t)((lbo >> 4) & 0x3fff) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3fff) << 32;
  d |= 1ull << 46;  // descriptor version of sm_100
  return d;         // base offset 0, layout type 0 (no swizzle)
}

// Instruction descriptor of kind::f16 with an fp32 accumulator, both
// operands K-major, M = 128.
__host__ __device__ inline uint32_t idesc_f16(int bf16, int n) {
  const uint32_t fmt = bf16 ? 1u : 0u;
  return (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accum)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 16 consecutive fp32 columns of this thread's tensor-memory lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Byte offset of element (row, col) of a rows x cols 16-bit matrix in the
// K-major core-matrix layout (col = K): chunk-major, then 8-row group.
__host__ __device__ inline uint32_t core_off(int row, int col, int rows) {
  return (uint32_t)((((col >> 3) * (rows >> 3) + (row >> 3)) * 8 + (row & 7)) * 16 + (col & 7) * 2);
}

// ------------------------------------------------------------ neighbour map
// Rule k's pair i joins input `in` to output `out`; nbr_out[out*K + k] = in
// and nbr_in[in*K + k] = out.  A rulebook from get_indice_pairs holds at most
// one pair per (output, k) and per (input, k).  Pairs naming rows outside
// [0, n_in) x [0, n_out) are ignored.
__global__ void spc_nbr_kernel(const int32_t* __restrict__ pairs, int64_t cap, int K,
                               const int32_t* __restrict__ num, int in_slot, int64_t n_in, int64_t n_out,
                               int32_t* __restrict__ nbr_out, int32_t* __restrict__ nbr_in) {
  const int k = blockIdx.y;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t cnt = min((int64_t)max(__ldg(num + k), 0), cap);
  if (i >= cnt) return;
  const int32_t in = __ldg(pairs + ((int64_t)k * 2 + in_slot) * cap + i);
  const int32_t out = __ldg(pairs + ((int64_t)k * 2 + (1 - in_slot)) * cap + i);
  if (BFB_BAD(in >= 0 && in < n_in && out >= 0 && out < n_out)) return;
  if (in < 0 || in >= n_in || out < 0 || out >= n_out) return;
  if (nbr_out) nbr_out[(int64_t)out * K + k] = in;
  if (nbr_in) nbr_in[(int64_t)in * K + k] = out;
}

// ------------------------------------------------------------ filter layouts
// Tensor-core operand B of offset k: an n x c matrix (n = output channel of
// this GEMM, c = reduced channel) in the core-matrix layout.  Forward: B(n, c)
// = filters[k][c][n]; transposed (input gradient): B(n, c) = filters[k][n][c].
template <class T>
__global__ void spc_prep_tc_kernel(const T* __restrict__ w, int K, int N, int Ck, int transposed,
                                   T* __restrict__ wp) {
  const int64_t total = (int64_t)K * N * Ck;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int k = (int)(e / ((int64_t)N * Ck));
    const int r = (int)(e - (int64_t)k * N * Ck);
    const int n = r / Ck, c = r - n * Ck;
    const T v = transposed ? w[((int64_t)k * N + n) * Ck + c] : w[((int64_t)k * Ck + c) * N + n];
    char* blk = reinterpret_cast<char*>(wp) + (size_t)k * N * Ck * sizeof(T);
    *reinterpret_cast<T*>(blk + core_off(n, c, N)) = v;
  }
}

// SIMT operand: fp32 [K][Ck][Npad], zero past N.
template <class T>
__global__ void spc_prep_simt_kernel(const T* __restrict__ w, int K, int N, int Ck, int Npad, int transposed,
                                     float* __restrict__ wp) {
  const int64_t total = (int64_t)K * Ck * Npad;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int k = (int)(e / ((int64_t)Ck * Npad));
    const int r = (int)(e - (int64_t)k * Ck * Npad);
    const int c = r / Npad, n = r - c * Npad;
    float v = 0.f;
    if (n < N) v = to_f32(transposed ? w[((int64_t)k * N + n) * Ck + c] : w[((int64_t)k * Ck + c) * N + n]);
    wp[e] = v;
  }
}

// Output epilogue shared by both convolution kernels: the reference adds the
// bias to the already rounded convolution output, so round twice.
template <class T>
__device__ __forceinline__ T epilogue(float acc, const T* bias, int n) {
  const T o = from_f32<T>(acc);
  if (!bias) return o;
  return from_f32<T>(to_f32(o) + to_f32(bias[n]));
}

// ---------------------------------------------------- tensor-core convolution
// One CTA per 128 destination rows.  x [n_src][Ck], nbr [n_dst][K],
// wp = spc_prep_tc_kernel's blocks, out [n_dst][N].  S pipeline stages: the
// rows of offsets j+1 .. j+S-1 are in flight while the tensor cores work on
// offset j.
template <class T, int S>
__global__ __launch_bounds__(kTcThreads) void spc_conv_tc_kernel(const T* __restrict__ x, int Ck,
                                                                 const int32_t* __restrict__ nbr, int K,
                                                                 int64_t n_dst, const T* __restrict__ wp, int N,
                                                                 uint32_t tmem_cols, const T* __restrict__ bias,
                                                                 T* __restrict__ out) {
  extern __shared__ __align__(1024) unsigned char smem[];
  __shared__ __align__(8) uint64_t bar_full[S];  // filter block of a stage has landed
  __shared__ __align__(8) uint64_t bar_mma[S];   // tensor cores are done with a stage
  __shared__ uint32_t s_tmem;
  __shared__ int s_act[kMaxK];
  __shared__ int s_nact;
  __shared__ uint32_t s_mask[(kMaxK + 31) / 32];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t row0 = (int64_t)blockIdx.x * kTcRows;
  const uint32_t a_bytes = (uint32_t)kTcRows * Ck * 2u, b_bytes = (uint32_t)N * Ck * 2u;
  // stage s: A rows at smem + s * (a + b), its filter block right after;
  // the tile's rows of the neighbour table after the stages
  auto st_a = [&](int s) { return smem + (size_t)s * (a_bytes + b_bytes); };
  auto st_b = [&](int s) { return smem + (size_t)s * (a_bytes + b_bytes) + a_bytes; };
  int32_t* s_nbr = reinterpret_cast<int32_t*>(smem + (size_t)S * (a_bytes + b_bytes));  // [128][K]

  if (tid < (kMaxK + 31) / 32) s_mask[tid] = 0u;
  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&bar_full[i], 1);
      mbar_init(&bar_mma[i], 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  __syncthreads();
  // the tile's neighbour rows: one contiguous slice of the table, read with
  // 16-byte loads (the slice starts on a 512-byte boundary); rows past n_dst
  // read as -1
  {
    const int64_t rows = min((int64_t)kTcRows, n_dst - row0);
    const int valid = (int)(rows * K), total = kTcRows * K;
    const int4* src4 = reinterpret_cast<const int4*>(nbr + row0 * K);
    int4* dst4 = reinterpret_cast<int4*>(s_nbr);
    for (int e4 = tid; e4 < total / 4; e4 += kTcThreads) {
      int4 v;
      if (e4 * 4 + 3 < valid) {
        v = __ldg(src4 + e4);
      } else {
        int t[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) t[i] = e4 * 4 + i < valid ? __ldg(nbr + row0 * K + e4 * 4 + i) : -1;
        v = make_int4(t[0], t[1], t[2], t[3]);
      }
      dst4[e4] = v;
    }
  }
  __syncthreads();
  {
    // the offsets any row of the tile uses: thread = row, one mask word of
    // 32 offsets at a time
    for (int w = 0; w * 32 < K; ++w) {
      uint32_t bits = 0u;
      for (int k = w * 32; k < min(K, w * 32 + 32); ++k)
        if (s_nbr[tid * K + k] >= 0) bits |= 1u << (k & 31);
      if (bits) atomicOr(&s_mask[w], bits);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  if (tid == 0) {
    int m = 0;
    for (int k = 0; k < K; ++k)
      if (s_mask[k >> 5] >> (k & 31) & 1u) s_act[m++] = k;
    s_nact = m;
  }
  __syncthreads();
  const int na = s_nact;
  const int chunks = Ck >> 3;  // 16-byte chunks per row
  const uint32_t lbo_a = (uint32_t)(kTcRows / 8) * 128u, lbo_b = (uint32_t)(N / 8) * 128u;
  const uint32_t idesc = idesc_f16(std::is_same<T, __nv_bfloat16>::value ? 1 : 0, N);
  bool ok = true;

  // Thread t stages all chunks of tile row t: in the core-matrix layout, row
  // r's chunk kc is the 16 bytes at (kc * 128 + r) * 16.  A row without a neighbour for the
  // offset must read as zeros; `dirty[s]` records whether this row of stage
  // s may hold data, so a row that is already zero is not rewritten (most
  // rows of a sparse tile have no neighbour for most offsets).
  bool dirty[S];
#pragma unroll
  for (int i = 0; i < S; ++i) dirty[i] = true;
  // Stage s = j % S holds offset j; its n-th use (n = j / S) completes
  // phase n of bar_full[s] and of bar_mma[s].  Iteration j loads offset
  // j + P into the stage last read by the MMAs of offset j + P - S: with
  // S >= 3, P = S - 2, so that stage was issued two iterations ago and its
  // MMAs have usually finished (S = 2: P = 1, the previous offset's).  Every
  // iteration commits one cp.async group (empty when nothing is left), so
  // "all but the newest P groups" is always offset j's rows.
  constexpr int P = S >= 3 ? S - 2 : 1;
  auto load_stage = [&](int j) {
    const int s = j % S;
    const int k = s_act[j];
    if (tid == 0) {
      mbar_expect_tx(&bar_full[s], b_bytes);
      bulk_g2s(st_b(s), wp + (size_t)k * N * Ck, b_bytes, &bar_full[s]);
    }
    const int32_t src = s_nbr[tid * K + k];
    bool d = false;
#pragma unroll
    for (int i = 0; i < S; ++i)
      if (i == s) d = dirty[i];
    if (src >= 0 || d) {
      const T* p = x + (src >= 0 ? (int64_t)src * Ck : 0);
      for (int kc = 0; kc < chunks; ++kc)
        cp_async16(st_a(s) + (size_t)(tid + kc * kTcThreads) * 16, p + (src >= 0 ? kc * 8 : 0), src >= 0);
#pragma unroll
      for (int i = 0; i < S; ++i)
        if (i == s) dirty[i] = src >= 0;
    }
  };

  for (int j = 0; j < P; ++j) {
    if (j < na) load_stage(j);
    cp_async_commit();
  }
  for (int j = 0; j < na; ++j) {
    const int s = j % S;
    const int jn = j + P;  // the offset loaded in this iteration
    if (jn < na) {
      const int prev = jn - S;  // the stage's previous offset
      if (prev >= 0 && !mbar_wait(&bar_mma[jn % S], (uint32_t)((prev / S) & 1))) ok = false;
      load_stage(jn);
    }
    cp_async_commit();
    cp_async_wait<P>();
    fence_async_smem();  // the cp.async rows become visible to the tensor cores
    __syncthreads();
    if (tid == 0) {
      if (!mbar_wait(&bar_full[s], (uint32_t)((j / S) & 1))) ok = false;
      tc_fence_after();
      const uint32_t a0 = smem_u32(st_a(s)), b0 = smem_u32(st_b(s));
      for (int t = 0; t < (Ck >> 4); ++t)
        umma_f16(tmem, smem_desc(a0 + t * 2 * lbo_a, lbo_a, 128u), smem_desc(b0 + t * 2 * lbo_b, lbo_b, 128u), idesc,
                 (j > 0 || t > 0) ? 1u : 0u);
      umma_commit(&bar_mma[s]);
    }
  }
  if (na > 0 && !mbar_wait(&bar_mma[(na - 1) % S], (uint32_t)(((na - 1) / S) & 1))) ok = false;
  cp_async_wait<0>();
  tc_fence_after();

  // epilogue: warp w owns tensor-memory lanes (tile rows) 32w .. 32w+31
  const int r = warp * 32 + lane;
  const int64_t row = row0 + r;
  for (int c0 = 0; c0 < N; c0 += 16) {
    float v[16];
    if (na > 0) {
      tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, v);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = 0.f;
    }
    if (row < n_dst) {
      __align__(16) T o[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) o[i] = epilogue<T>(ok ? v[i] : 0.f, bias, c0 + i);
      uint4* dst = reinterpret_cast<uint4*>(out + row * N + c0);
      dst[0] = *reinterpret_cast<const uint4*>(&o[0]);
      dst[1] = *reinterpret_cast<const uint4*>(&o[8]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tmem_cols) : "memory");
}

// ------------------------------------------------------------ SIMT convolution
// Rule-major: one launch per kernel offset k, in ascending order.  A block
// takes 64 of rule k's pairs at a time (every row useful), stages their
// source rows and filter k in shared memory (32 reduced channels per step),
// and each thread forms 4 pairs x 4 output channels per 64-column pass of
// the dot products x[src] @ filters[k] (fp32 FMA, ascending reduced
// channel), then adds them to the fp32 accumulator rows acc[dst] (read,
// add, write: a rule names every destination row at most once and the rules
// run one after another, so no atomics; an output is the rule-ordered sum of
// per-rule dot products, as the reference's matmul-then-index_add_ forms
// it).  NP 64-column passes per block; blockIdx.y picks the column group.
template <class T, int NP>
__global__ __launch_bounds__(kSimtThreads) void spc_rule_kernel(const T* __restrict__ x, int Ck,
                                                                const int32_t* __restrict__ pairs, int64_t cap,
                                                                const int32_t* __restrict__ num, int k, int src_slot,
                                                                int64_t n_src, int64_t n_dst,
                                                                const float* __restrict__ wp, int N, int Npad,
                                                                float* __restrict__ acc) {
  __shared__ __align__(16) float s_a[kSimtChunk][64 + 4];  // [channel][pair], padded
  __shared__ __align__(16) float s_w[kSimtChunk][NP * 64];
  __shared__ int32_t s_src[64], s_dst[64];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int n0 = blockIdx.y * NP * 64;
  const int64_t cnt = min((int64_t)max(__ldg(num + k), 0), cap);
  const int32_t* ps = pairs + ((int64_t)k * 2 + src_slot) * cap;
  const int32_t* pd = pairs + ((int64_t)k * 2 + (1 - src_slot)) * cap;
  for (int64_t t0 = (int64_t)blockIdx.x * 64; t0 < cnt; t0 += (int64_t)gridDim.x * 64) {
    if (tid < 64) {
      const int64_t p = t0 + tid;
      int32_t a = -1, b = -1;
      if (p < cnt) {
        a = __ldg(ps + p);
        b = __ldg(pd + p);
        if (BFB_BAD(a >= 0 && a < n_src && b >= 0 && b < n_dst)) a = b = -1;
        if (a < 0 || a >= n_src || b < 0 || b >= n_dst) a = b = -1;
      }
      s_src[tid] = a;
      s_dst[tid] = b;
    }
    __syncthreads();
    float r[NP][4][4];
#pragma unroll
    for (int q = 0; q < NP; ++q)
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int c = 0; c < 4; ++c) r[q][i][c] = 0.f;
    for (int c0 = 0; c0 < Ck; c0 += kSimtChunk) {
      const int cw = min(kSimtChunk, Ck - c0);
      for (int e = tid; e < 64 * kSimtChunk; e += kSimtThreads) {
        const int pp = e / kSimtChunk, c = e - pp * kSimtChunk;
        const int32_t a = s_src[pp];
        s_a[c][pp] = (a >= 0 && c < cw) ? to_f32(x[(int64_t)a * Ck + c0 + c]) : 0.f;
      }
      for (int e = tid; e < kSimtChunk * NP * 64; e += kSimtThreads) {
        const int c = e / (NP * 64), n = e - c * (NP * 64);
        s_w[c][n] = (c < cw && n0 + n < Npad) ? wp[((int64_t)k * Ck + c0 + c) * Npad + n0 + n] : 0.f;
      }
      __syncthreads();
      for (int c = 0; c < cw; ++c) {
        const float4 a4 = *reinterpret_cast<const float4*>(&s_a[c][ty * 4]);
        const float av[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
        for (int q = 0; q < NP; ++q) {
          const float4 w4 = *reinterpret_cast<const float4*>(&s_w[c][q * 64 + tx * 4]);
          const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int u = 0; u < 4; ++u) r[q][i][u] = fmaf(av[i], wv[u], r[q][i][u]);
        }
      }
      __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int32_t d = s_dst[ty * 4 + i];
      if (d < 0) continue;
      float* arow = acc + (int64_t)d * N;
#pragma unroll
      for (int q = 0; q < NP; ++q)
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int n = n0 + q * 64 + tx * 4 + u;
          if (n < N) arow[n] += r[q][i][u];
        }
    }
    __syncthreads();  // s_src / s_dst are rewritten next
  }
}

// out = epilogue(acc) over [rows][N] (the fp32 sums rounded once, + bias).
template <class T>
__global__ void spc_finish_kernel(const float* __restrict__ acc, int64_t rows, int N, const T* __restrict__ bias,
                                  T* __restrict__ out) {
  const int64_t total = rows * N;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x)
    out[e] = epilogue<T>(acc[e], bias, (int)(e % N));
}

// ------------------------------------------------------------ filter gradient
// The pairs of every rule are cut into chunks of one common length L
// (a multiple of 32) chosen so that all chunks fit `slots` partial buffers:
// rule k gets ceil(n_k / L) chunks, numbered from cpre[k].  Planned on the
// device from the rule counts, so the host reads nothing; the result depends
// only on the counts, so the sum order is fixed.
struct DwPlan {
  int32_t L;
  int32_t cpre[kMaxK + 1];
};

__global__ void spc_dw_plan_kernel(const int32_t* __restrict__ num, int K, int64_t cap, int slots,
                                   DwPlan* __restrict__ plan) {
  // one warp: the counts are loaded in parallel, the prefix is a warp scan
  const int lane = threadIdx.x & 31;
  if (threadIdx.x >= 32) return;
  int64_t total = 0;
  for (int k = lane; k < K; k += 32) total += min((int64_t)max(__ldg(num + k), 0), cap);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
  const int64_t room = max(slots - K, 1);
  const int64_t L = max((int64_t)32, ((total + room - 1) / room + 31) / 32 * 32);
  int32_t carry = 0;
  for (int k0 = 0; k0 < K; k0 += 32) {
    const int k = k0 + lane;
    const int32_t c = k < K ? (int32_t)((min((int64_t)max(__ldg(num + k), 0), cap) + L - 1) / L) : 0;
    int32_t x = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (k < K) plan->cpre[k] = carry + x - c;
    carry += __shfl_sync(0xffffffffu, x, 31);
  }
  if (lane == 0) {
    plan->cpre[K] = carry;
    plan->L = (int32_t)L;
  }
}

// Block (slot, tile): the slot's chunk of one rule, a 64 x 64 tile (input
// channel x output channel) of sum_p x[in_p][ci] * g[out_p][co] in fp32,
// written to part[slot][ci][co].  Slots past the last chunk do nothing.
template <class T>
__global__ __launch_bounds__(kSimtThreads) void spc_dw_kernel(const T* __restrict__ x, int Cin,
                                                              const T* __restrict__ g, int Cout,
                                                              const int32_t* __restrict__ pairs, int64_t cap,
                                                              const int32_t* __restrict__ num, int K, int in_slot,
                                                              int64_t n_in, int64_t n_out,
                                                              const DwPlan* __restrict__ plan, int tiles_co,
                                                              float* __restrict__ part) {
  __shared__ __align__(16) float s_x[kSimtChunk][64];
  __shared__ __align__(16) float s_g[kSimtChunk][64];
  __shared__ int32_t s_pi[kSimtChunk], s_po[kSimtChunk];
  const int slot = blockIdx.x;
  if (slot >= plan->cpre[K]) return;
  int k = 0;
  while (k + 1 < K && plan->cpre[k + 1] <= slot) ++k;
  const int64_t L = plan->L;
  const int ti = blockIdx.y / tiles_co, tc = blockIdx.y - ti * tiles_co;
  const int ci0 = ti * 64, co0 = tc * 64;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t cnt = min((int64_t)max(__ldg(num + k), 0), cap);
  const int64_t p0 = (int64_t)(slot - plan->cpre[k]) * L, p1 = min(cnt, p0 + L);
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[i][q] = 0.f;
  for (int64_t pb = p0; pb < p1; pb += kSimtChunk) {
    const int pw = (int)min((int64_t)kSimtChunk, p1 - pb);
    if (tid < kSimtChunk) {
      int32_t a = -1, b = -1;
      if (tid < pw) {
        a = __ldg(pairs + ((int64_t)k * 2 + in_slot) * cap + pb + tid);
        b = __ldg(pairs + ((int64_t)k * 2 + (1 - in_slot)) * cap + pb + tid);
        if (BFB_BAD(a >= 0 && a < n_in && b >= 0 && b < n_out)) a = b = -1;
        if (a < 0 || a >= n_in || b < 0 || b >= n_out) a = b = -1;
      }
      s_pi[tid] = a;
      s_po[tid] = b;
    }
    __syncthreads();
    for (int e = tid; e < kSimtChunk * 64; e += kSimtThreads) {
      const int p = e >> 6, c = e & 63;
      const int32_t a = s_pi[p], b = s_po[p];
      s_x[p][c] = (a >= 0 && ci0 + c < Cin) ? to_f32(x[(int64_t)a * Cin + ci0 + c]) : 0.f;
      s_g[p][c] = (b >= 0 && co0 + c < Cout) ? to_f32(g[(int64_t)b * Cout + co0 + c]) : 0.f;
    }
    __syncthreads();
    for (int p = 0; p < pw; ++p) {
      const float4 a = *reinterpret_cast<const float4*>(&s_x[p][ty * 4]);
      const float4 b = *reinterpret_cast<const float4*>(&s_g[p][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[i][q] = fmaf(av[i], bv[q], acc[i][q]);
    }
    __syncthreads();
  }
  float* dst = part + (int64_t)slot * Cin * Cout;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int ci = ci0 + ty * 4 + i;
    if (ci >= Cin) continue;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int co = co0 + tx * 4 + q;
      if (co < Cout) dst[(int64_t)ci * Cout + co] = acc[i][q];
    }
  }
}

// Tensor-core form of spc_dw_kernel (fp16 / bf16, Cin <= 128 and a multiple
// of 8, Cout a multiple of 16 up to 256): the partial of a chunk is
// D[ci][co] = sum_p x[in_p][ci] * g[out_p][co], one tcgen05 GEMM chain with
// M = 128 (input channels, zero past Cin), N = Cout and the pairs as the
// reduction dimension, 128 pairs per stage.  Both operands are MN-major: a
// core matrix is 8 pairs x 16 bytes of one row chunk, so every gathered
// 16-byte chunk of an input or gradient row is copied (cp.async) straight to
// its place.
__device__ __forceinline__ uint32_t mn_off(int p, int c8, int groups) {
  return (uint32_t)((((p >> 3) * groups + c8) * 8 + (p & 7)) * 16);
}

template <class T>
__global__ __launch_bounds__(kTcThreads) void spc_dw_tc_kernel(const T* __restrict__ x, int Cin,
                                                               const T* __restrict__ g, int Cout,
                                                               const int32_t* __restrict__ pairs, int64_t cap,
                                                               const int32_t* __restrict__ num, int K, int in_slot,
                                                               int64_t n_in, int64_t n_out,
                                                               const DwPlan* __restrict__ plan, uint32_t tmem_cols,
                                                               float* __restrict__ part) {
  extern __shared__ __align__(1024) unsigned char smem[];
  __shared__ __align__(8) uint64_t bar_mma[2];
  __shared__ uint32_t s_tmem;
  const int slot = blockIdx.x;
  if (slot >= plan->cpre[K]) return;  // uniform, before any allocation
  int k = 0;
  while (k + 1 < K && plan->cpre[k + 1] <= slot) ++k;
  const int64_t L = plan->L;
  const int64_t cnt = min((int64_t)max(__ldg(num + k), 0), cap);
  const int64_t p0 = (int64_t)(slot - plan->cpre[k]) * L, p1 = min(cnt, p0 + L);
  const int nst = p1 > p0 ? (int)((p1 - p0 + kTcRows - 1) / kTcRows) : 0;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t a_bytes = (uint32_t)kTcRows * kTcRows * 2u, b_bytes = (uint32_t)Cout * kTcRows * 2u;
  auto st_a = [&](int s) { return smem + (size_t)s * (a_bytes + b_bytes); };
  auto st_b = [&](int s) { return smem + (size_t)s * (a_bytes + b_bytes) + a_bytes; };
  // channel rows past Cin are never loaded: zero both A stages once
  for (int e = tid; e < (int)(2 * (a_bytes + b_bytes) / 16); e += kTcThreads)
    reinterpret_cast<uint4*>(smem)[e] = make_uint4(0u, 0u, 0u, 0u);
  if (tid == 0) {
    mbar_init(&bar_mma[0], 1);
    mbar_init(&bar_mma[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  const int ci8 = Cin >> 3, co8 = Cout >> 3;
  const uint32_t lbo_a = (uint32_t)(kTcRows / 8) * 128u, lbo_b = (uint32_t)co8 * 128u;
  const uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  const uint32_t idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | (1u << 15) | (1u << 16) |
                         ((uint32_t)(Cout >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);
  bool ok = true;

  // thread t gathers pair t of the step: its input row's chunks into A,
  // its output-gradient row's chunks into B (zeros past the chunk's end)
  auto load_step = [&](int j) {
    const int s = j & 1;
    const int64_t p = p0 + (int64_t)j * kTcRows + tid;
    int32_t a = -1, b = -1;
    if (p < p1) {
      a = __ldg(pairs + ((int64_t)k * 2 + in_slot) * cap + p);
      b = __ldg(pairs + ((int64_t)k * 2 + (1 - in_slot)) * cap + p);
      if (BFB_BAD(a >= 0 && a < n_in && b >= 0 && b < n_out)) a = b = -1;
      if (a < 0 || a >= n_in || b < 0 || b >= n_out) a = b = -1;
    }
    const T* xa = x + (a >= 0 ? (int64_t)a * Cin : 0);
    const T* gb = g + (b >= 0 ? (int64_t)b * Cout : 0);
    for (int c = 0; c < ci8; ++c) cp_async16(st_a(s) + mn_off(tid, c, kTcRows / 8), xa + (a >= 0 ? c * 8 : 0), a >= 0);
    for (int c = 0; c < co8; ++c) cp_async16(st_b(s) + mn_off(tid, c, co8), gb + (b >= 0 ? c * 8 : 0), b >= 0);
  };

  if (nst > 0) load_step(0);
  cp_async_commit();
  for (int j = 0; j < nst; ++j) {
    const int s = j & 1;
    if (j + 1 < nst) {
      if (j >= 1 && !mbar_wait(&bar_mma[s ^ 1], (uint32_t)(((j - 1) >> 1) & 1))) ok = false;
      load_step(j + 1);
    }
    cp_async_commit();
    cp_async_wait<1>();
    fence_async_smem();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint32_t a0 = smem_u32(st_a(s)), b0 = smem_u32(st_b(s));
      for (int t = 0; t < kTcRows / 16; ++t)
        umma_f16(tmem, smem_desc(a0 + t * 2 * lbo_a, lbo_a, 128u), smem_desc(b0 + t * 2 * lbo_b, lbo_b, 128u), idesc,
                 (j > 0 || t > 0) ? 1u : 0u);
      umma_commit(&bar_mma[s]);
    }
  }
  if (nst > 0 && !mbar_wait(&bar_mma[(nst - 1) & 1], (uint32_t)(((nst - 1) >> 1) & 1))) ok = false;
  cp_async_wait<0>();
  tc_fence_after();

  // epilogue: lane = input channel, columns = output channels
  const int ci = warp * 32 + lane;
  float* dst = part + (int64_t)slot * Cin * Cout + (int64_t)ci * Cout;
  for (int c0 = 0; c0 < Cout; c0 += 16) {
    float v[16];
    if (nst > 0) {
      tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, v);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = 0.f;
    }
    if (ci < Cin) {
#pragma unroll
      for (int i = 0; i < 16; i += 4)
        *reinterpret_cast<float4*>(dst + c0 + i) =
            make_float4(ok ? v[i] : 0.f, ok ? v[i + 1] : 0.f, ok ? v[i + 2] : 0.f, ok ? v[i + 3] : 0.f);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tmem_cols) : "memory");
}

// dw[k] = sum of rule k's chunk partials (0 for a rule without pairs).  A
// block covers 32 consecutive entries of dw[k] (lanes, coalesced) and 8
// chunk groups (warps): warp w adds chunks w, w + 8, ... in order, then the
// 8 group sums are added in group order -- a fixed tree, so the result is
// deterministic, and one rule's hundreds of chunks are summed 8-wide.
template <class T>
__global__ __launch_bounds__(256) void spc_dw_reduce_kernel(const float* __restrict__ part, int K,
                                                            const DwPlan* __restrict__ plan, int64_t cc,
                                                            T* __restrict__ dw) {
  __shared__ float s_sum[8][33];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int k = blockIdx.y;
  const int64_t r = (int64_t)blockIdx.x * 32 + lane;
  const int c0 = plan->cpre[k], c1 = plan->cpre[k + 1];
  float s = 0.f;
  if (r < cc) {
    int c = c0 + w;
    for (; c + 24 < c1; c += 32) {  // four loads in flight, added in order
      float v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = __ldg(part + (int64_t)(c + 8 * u) * cc + r);
#pragma unroll
      for (int u = 0; u < 4; ++u) s += v[u];
    }
    for (; c < c1; c += 8) s += __ldg(part + (int64_t)c * cc + r);
  }
  s_sum[w][lane] = s;
  __syncthreads();
  if (w == 0 && r < cc) {
    float t = 0.f;
#pragma unroll
    for (int g = 0; g < 8; ++g) t += s_sum[g][lane];
    dw[(int64_t)k * cc + r] = from_f32<T>(t);
  }
}

// ------------------------------------------------------------ max pooling
template <class T>
__global__ void spc_maxpool_kernel(const T* __restrict__ x, int C, const int32_t* __restrict__ nbr, int K,
                                   int64_t n_out, T* __restrict__ out) {
  const int64_t total = n_out * C;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = e / C;
    const int c = (int)(e - o * C);
    T m = from_f32<T>(0.f);  // the reference pools into zeros with include_self
    for (int k = 0; k < K; ++k) {
      const int32_t i = __ldg(nbr + o * K + k);
      if (i >= 0) {
        const T v = x[(int64_t)i * C + c];
        if (to_f32(v) > to_f32(m)) m = v;
      }
    }
    out[e] = m;
  }
}

// Input-stationary: the gradient of input i sums, in ascending offset, the
// output gradients of the outputs whose pooled value equals x[i] (all equal
// maxima receive it), rounded to T after every add as the reference's
// index_add_ into a T tensor does.
template <class T>
__global__ void spc_maxpool_bwd_kernel(const T* __restrict__ x, const T* __restrict__ y, const T* __restrict__ gy,
                                       int C, const int32_t* __restrict__ nbr_in, int K, int64_t n_in,
                                       T* __restrict__ gx) {
  const int64_t total = n_in * C;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = e / C;
    const int c = (int)(e - i * C);
    const float xv = to_f32(x[e]);
    T s = from_f32<T>(0.f);
    for (int k = 0; k < K; ++k) {
      const int32_t o = __ldg(nbr_in + i * K + k);
      if (o >= 0 && to_f32(y[(int64_t)o * C + c]) == xv) s = from_f32<T>(to_f32(s) + to_f32(gy[(int64_t)o * C + c]));
    }
    gx[e] = s;
  }
}

// ------------------------------------------------------------------ host side
struct ConvWork {
  int32_t* nbr_out = nullptr;  // [n_dst][K]
  int32_t* nbr_in = nullptr;   // [n_in][K] (backward)
  void* wprep = nullptr;       // forward-direction filter operand
  void* wprep_t = nullptr;     // transposed filter operand (backward)
  float* part = nullptr;       // filter-gradient partials
  DwPlan* dwplan = nullptr;
  float* acc = nullptr;        // fp32 sums of the rule-major path (16-bit features)
};

bool tc_ok(int dtype, int64_t Ck, int64_t N, int64_t K) {
  if (dtype != BFB_F16 && dtype != BFB_BF16) return false;
  if (Ck % 16 || N % 16 || Ck < 16 || N < 16 || N > 256) return false;
  const size_t smem = 2 * ((size_t)kTcRows * Ck * 2 + (size_t)N * Ck * 2) + (size_t)kTcRows * K * 4;
  return smem <= 200 * 1024;
}

// Room for either filter operand (the fp32 SIMT one is the larger), so the
// path can be chosen per call (e.g. by pointer alignment).
size_t prep_bytes(int64_t K, int64_t Ck, int64_t N) {
  return (size_t)K * Ck * ceil_div(N, 4) * 4 * sizeof(float);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Partial buffers of the filter gradient: up to 1024, at most 64 MiB.
int dw_slots(int64_t K, int64_t Cin, int64_t Cout) {
  const int64_t fit = (64ll << 20) / (Cin * Cout * (int64_t)sizeof(float));
  return (int)std::max<int64_t>(K + 1, std::min<int64_t>(1024, fit));
}

size_t carve_conv(void* base, int dtype, int64_t n_in, int64_t n_out, int64_t K, int64_t cin, int64_t cout,
                  int64_t cap, int backward, ConvWork* w) {
  Carver c(base);
  w->nbr_out = c.take<int32_t>((size_t)(n_out * K));
  w->wprep = c.take<char>(prep_bytes(K, cin, cout));
  if (dtype != BFB_F32) w->acc = c.take<float>((size_t)std::max(n_out * cout, backward ? n_in * cin : 0));
  if (backward) {
    w->nbr_in = c.take<int32_t>((size_t)(n_in * K));
    w->wprep_t = c.take<char>(prep_bytes(K, cout, cin));
    w->part = c.take<float>((size_t)dw_slots(K, cin, cout) * cin * cout);
    w->dwplan = c.take<DwPlan>(1);
  }
  return c.bytes();
}

unsigned grid_for(int64_t total, int threads) {
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>(ceil_div(total, threads), 148 * 16));
}

int build_tables(const int32_t* pairs, int64_t K, int64_t cap, const int32_t* num, int in_slot, int64_t n_in,
                 int64_t n_out, int32_t* nbr_out, int32_t* nbr_in, cudaStream_t st) {
  if (nbr_out) BFB_CUDA(cudaMemsetAsync(nbr_out, 0xff, sizeof(int32_t) * (size_t)(n_out * K), st));
  if (nbr_in) BFB_CUDA(cudaMemsetAsync(nbr_in, 0xff, sizeof(int32_t) * (size_t)(n_in * K), st));
  if (cap > 0) {
    spc_nbr_kernel<<<dim3((unsigned)ceil_div(cap, 256), (unsigned)K), 256, 0, st>>>(pairs, cap, (int)K, num, in_slot,
                                                                                    n_in, n_out, nbr_out, nbr_in);
    BFB_CHECK_LAUNCH();
  }
  return BFB_OK;
}

template <class T>
bool use_tc(int64_t Ck, int64_t N, int64_t K, const void* x, const void* out, const void* wprep) {
  if constexpr (std::is_same<T, float>::value) {
    return false;
  } else {
    const int dtype = std::is_same<T, __half>::value ? BFB_F16 : BFB_BF16;
    return tc_ok(dtype, Ck, N, K) && aligned16(x) && aligned16(out) && aligned16(wprep);
  }
}

// Tensor-core path over the neighbour table nbr [n_dst][K].
template <class T>
int launch_conv_tc(const T* x, int64_t Ck, const int32_t* nbr, int64_t K, int64_t n_dst, const T* w, int64_t N,
                   int transposed, const T* bias, void* wprep, T* out, cudaStream_t st) {
  if constexpr (!std::is_same<T, float>::value) {
    T* wp = static_cast<T*>(wprep);
    spc_prep_tc_kernel<T><<<grid_for(K * N * Ck, 256), 256, 0, st>>>(w, (int)K, (int)N, (int)Ck, transposed, wp);
    BFB_CHECK_LAUNCH();
    uint32_t cols = 32;
    while (cols < (uint32_t)N) cols <<= 1;
    const size_t stage = (size_t)kTcRows * Ck * 2 + (size_t)N * Ck * 2;
    // two stages: measured faster than three or four here, because more
    // blocks fit on an SM (the tile's latency is hidden across blocks)
    size_t smem = 2 * stage + (size_t)kTcRows * K * 4;
    // at most 512 / cols blocks per SM, so that every resident block's
    // tensor-memory allocation succeeds at once
    const size_t per_sm = 227 * 1024, min_smem = per_sm / (512 / cols + 1) + 1;
    smem = std::max(smem, min_smem);
    BFB_CUDA(cudaFuncSetAttribute(spc_conv_tc_kernel<T, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    spc_conv_tc_kernel<T, 2><<<(unsigned)ceil_div(n_dst, kTcRows), kTcThreads, smem, st>>>(
        x, (int)Ck, nbr, (int)K, n_dst, wp, (int)N, cols, bias, out);
    BFB_CHECK_LAUNCH();
    return BFB_OK;
  } else {
    return BFB_ERR_UNSUPPORTED_DTYPE;
  }
}

// Rule-major FMA path straight over the rulebook: pair slot src_slot names
// the source row (of x, n_src rows), the other slot the destination row.
template <class T>
int launch_conv_rules(const T* x, int64_t Ck, const int32_t* pairs, int64_t cap, const int32_t* num, int64_t K,
                      int src_slot, int64_t n_src, int64_t n_dst, const T* w, int64_t N, int transposed,
                      const T* bias, void* wprep, float* acc_ws, T* out, cudaStream_t st) {
  const int64_t Npad = ceil_div(N, 4) * 4;
  float* wp = static_cast<float*>(wprep);
  spc_prep_simt_kernel<T><<<grid_for(K * Ck * Npad, 256), 256, 0, st>>>(w, (int)K, (int)N, (int)Ck, (int)Npad,
                                                                        transposed, wp);
  BFB_CHECK_LAUNCH();
  constexpr bool f32 = std::is_same<T, float>::value;
  float* acc = f32 ? reinterpret_cast<float*>(out) : acc_ws;
  BFB_CUDA(cudaMemsetAsync(acc, 0, sizeof(float) * (size_t)(n_dst * N), st));
  if (cap > 0) {
    const int np = Npad <= 64 ? 1 : Npad <= 128 ? 2 : 4;
    const dim3 grid((unsigned)std::min<int64_t>(ceil_div(cap, 64), 148 * 4), (unsigned)ceil_div(Npad, np * 64));
    for (int64_t k = 0; k < K; ++k) {
      if (np == 1)
        spc_rule_kernel<T, 1><<<grid, kSimtThreads, 0, st>>>(x, (int)Ck, pairs, cap, num, (int)k, src_slot, n_src,
                                                             n_dst, wp, (int)N, (int)Npad, acc);
      else if (np == 2)
        spc_rule_kernel<T, 2><<<grid, kSimtThreads, 0, st>>>(x, (int)Ck, pairs, cap, num, (int)k, src_slot, n_src,
                                                             n_dst, wp, (int)N, (int)Npad, acc);
      else
        spc_rule_kernel<T, 4><<<grid, kSimtThreads, 0, st>>>(x, (int)Ck, pairs, cap, num, (int)k, src_slot, n_src,
                                                             n_dst, wp, (int)N, (int)Npad, acc);
      BFB_CHECK_LAUNCH();
    }
  }
  if (!f32 || bias) {
    spc_finish_kernel<T><<<grid_for(n_dst * N, 256), 256, 0, st>>>(acc, n_dst, (int)N, bias, out);
    BFB_CHECK_LAUNCH();
  }
  return BFB_OK;
}

int check_conv_args(int dtype, int64_t n_in, int64_t cin, int64_t K, int64_t cout, int64_t cap, int64_t n_out) {
  if (!dtype_size(dtype)) return BFB_ERR_UNSUPPORTED_DTYPE;
  if (n_in < 0 || n_out < 0 || cap < 0 || cin <= 0 || cout <= 0 || K <= 0) return BFB_ERR_INVALID_ARG;
  if (K > kMaxK) return BFB_ERR_INVALID_ARG;
  if (n_in * K >= 0x7fffffffLL || n_out * K >= 0x7fffffffLL || n_in >= 0x7fffffffLL) return BFB_ERR_TOO_LARGE;
  return BFB_OK;
}

template <class T>
int conv_forward(const void* features, int64_t n_in, int64_t cin, const void* filters, int64_t K, int64_t cout,
                 const int32_t* pairs, int64_t cap, const int32_t* num, int64_t n_out, int inverse, const void* bias,
                 void* out, const ConvWork& w, cudaStream_t st) {
  if (n_out == 0) return BFB_OK;
  const int in_slot = inverse ? 1 : 0;
  const T* x = static_cast<const T*>(features);
  if (use_tc<T>(cin, cout, K, features, out, w.wprep)) {
    BFB_TRY(build_tables(pairs, K, cap, num, in_slot, n_in, n_out, w.nbr_out, nullptr, st));
    return launch_conv_tc<T>(x, cin, w.nbr_out, K, n_out, static_cast<const T*>(filters), cout, 0,
                             static_cast<const T*>(bias), w.wprep, static_cast<T*>(out), st);
  }
  return launch_conv_rules<T>(x, cin, pairs, cap, num, K, in_slot, n_in, n_out, static_cast<const T*>(filters), cout,
                              0, static_cast<const T*>(bias), w.wprep, w.acc, static_cast<T*>(out), st);
}

template <class T>
int conv_backward(const void* features, int64_t n_in, int64_t cin, const void* filters, int64_t K, int64_t cout,
                  const void* out_bp, int64_t n_out, const int32_t* pairs, int64_t cap, const int32_t* num,
                  int inverse, void* input_grad, void* filters_grad, const ConvWork& w, cudaStream_t st) {
  const int in_slot = inverse ? 1 : 0;
  // input gradient: destination = inputs, source = output gradients,
  // reduced channel = cout, filters transposed
  const T* g = static_cast<const T*>(out_bp);
  if (n_in > 0) {
    if (use_tc<T>(cout, cin, K, out_bp, input_grad, w.wprep_t)) {
      BFB_TRY(build_tables(pairs, K, cap, num, in_slot, n_in, n_out, nullptr, w.nbr_in, st));
      BFB_TRY(launch_conv_tc<T>(g, cout, w.nbr_in, K, n_in, static_cast<const T*>(filters), cin, 1, nullptr,
                                w.wprep_t, static_cast<T*>(input_grad), st));
    } else {
      BFB_TRY(launch_conv_rules<T>(g, cout, pairs, cap, num, K, 1 - in_slot, n_out, n_in,
                                   static_cast<const T*>(filters), cin, 1, nullptr, w.wprep_t, w.acc,
                                   static_cast<T*>(input_grad), st));
    }
  }
  const int slots = dw_slots(K, cin, cout);
  spc_dw_plan_kernel<<<1, 32, 0, st>>>(num, (int)K, cap, slots, w.dwplan);
  BFB_CHECK_LAUNCH();
  bool tc = false;
  if constexpr (!std::is_same<T, float>::value)
    tc = cin <= kTcRows && cin % 8 == 0 && cout % 16 == 0 && cout >= 16 && cout <= 256 && aligned16(features) &&
         aligned16(out_bp);
  if constexpr (!std::is_same<T, float>::value) {
    if (tc) {
      uint32_t cols = 32;
      while (cols < (uint32_t)cout) cols <<= 1;
      const size_t per_sm = 227 * 1024, min_smem = per_sm / (512 / cols + 1) + 1;
      const size_t smem = std::max((size_t)2 * ((size_t)kTcRows * kTcRows * 2 + (size_t)cout * kTcRows * 2), min_smem);
      BFB_CUDA(cudaFuncSetAttribute(spc_dw_tc_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      spc_dw_tc_kernel<T><<<(unsigned)slots, kTcThreads, smem, st>>>(
          static_cast<const T*>(features), (int)cin, static_cast<const T*>(out_bp), (int)cout, pairs, cap, num, (int)K,
          in_slot, n_in, n_out, w.dwplan, cols, w.part);
      BFB_CHECK_LAUNCH();
    }
  }
  const int tiles_ci = (int)ceil_div(cin, 64), tiles_co = (int)ceil_div(cout, 64);
  if (!tc) {
    spc_dw_kernel<T><<<dim3((unsigned)slots, (unsigned)(tiles_ci * tiles_co)), kSimtThreads, 0, st>>>(
        static_cast<const T*>(features), (int)cin, static_cast<const T*>(out_bp), (int)cout, pairs, cap, num, (int)K,
        in_slot, n_in, n_out, w.dwplan, tiles_co, w.part);
    BFB_CHECK_LAUNCH();
  }
  spc_dw_reduce_kernel<T><<<dim3((unsigned)ceil_div(cin * cout, 32), (unsigned)K), 256, 0, st>>>(
      w.part, (int)K, w.dwplan, cin * cout, static_cast<T*>(filters_grad));
  BFB_CHECK_LAUNCH();
  return BFB_OK;
}

}  // namespace

int spconv_timeouts(uint64_t* out, int reset) {
  unsigned long long x = 0;
  BFB_CUDA(cudaMemcpyFromSymbol(&x, g_spc_timeouts, sizeof(x)));
  if (out) *out = x;
  if (reset) {
    const unsigned long long z = 0;
    BFB_CUDA(cudaMemcpyToSymbol(g_spc_timeouts, &z, sizeof(z)));
  }
  return BFB_OK;
}

}  // namespace bfb

using namespace bfb;

extern "C" int bfb_indice_conv_workspace_size(int64_t n_in, int64_t n_out, int64_t K, int64_t cin, int64_t cout,
                                              int64_t pair_cap, int dtype, int backward, size_t* bytes) {
  if (!bytes) return BFB_ERR_INVALID_ARG;
  BFB_TRY(check_conv_args(dtype, n_in, cin, K, cout, pair_cap, n_out));
  ConvWork w;
  *bytes = carve_conv(nullptr, dtype, n_in, n_out, K, cin, cout, pair_cap, backward, &w);
  return BFB_OK;
}

extern "C" int bfb_indice_conv(const void* features, int dtype, int64_t n_in, int64_t cin, const void* filters,
                               int64_t K, int64_t cout, const int32_t* indice_pairs, int64_t pair_cap,
                               const int32_t* indice_num, int64_t n_out, int inverse, const void* bias, void* out,
                               void* workspace, size_t workspace_bytes, void* stream) {
  BFB_INJECT_POINT();
  BFB_TRY(check_conv_args(dtype, n_in, cin, K, cout, pair_cap, n_out));
  if ((n_in > 0 && !features) || !filters || (pair_cap > 0 && (!indice_pairs || !indice_num)) || (n_out > 0 && !out))
    return BFB_ERR_INVALID_ARG;
  ConvWork w;
  if (carve_conv(nullptr, dtype, n_in, n_out, K, cin, cout, pair_cap, 0, &w) > workspace_bytes || !workspace)
    return BFB_ERR_WORKSPACE;
  carve_conv(workspace, dtype, n_in, n_out, K, cin, cout, pair_cap, 0, &w);
  cudaStream_t st = as_stream(stream);
  switch (dtype) {
    case BFB_F32:
      return conv_forward<float>(features, n_in, cin, filters, K, cout, indice_pairs, pair_cap, indice_num, n_out,
                                 inverse, bias, out, w, st);
    case BFB_F16:
      return conv_forward<__half>(features, n_in, cin, filters, K, cout, indice_pairs, pair_cap, indice_num, n_out,
                                  inverse, bias, out, w, st);
    case BFB_BF16:
      return conv_forward<__nv_bfloat16>(features, n_in, cin, filters, K, cout, indice_pairs, pair_cap, indice_num,
                                         n_out, inverse, bias, out, w, st);
    default:
      return BFB_ERR_UNSUPPORTED_DTYPE;
  }
}

extern "C" int bfb_indice_conv_backward(const void* features, int dtype, int64_t n_in, int64_t cin,
                                        const void* filters, int64_t K, int64_t cout, const void* out_bp,
                                        int64_t n_out, const int32_t* indice_pairs, int64_t pair_cap,
                                        const int32_t* indice_num, int inverse, void* input_grad,
                                        void* filters_grad, void* workspace, size_t workspace_bytes, void* stream) {
  BFB_INJECT_POINT();
  BFB_TRY(check_conv_args(dtype, n_in, cin, K, cout, pair_cap, n_out));
  if ((n_in > 0 && (!features || !input_grad)) || !filters || !filters_grad || (n_out > 0 && !out_bp) ||
      (pair_cap > 0 && (!indice_pairs || !indice_num)))
    return BFB_ERR_INVALID_ARG;
  ConvWork w;
  if (carve_conv(nullptr, dtype, n_in, n_out, K, cin, cout, pair_cap, 1, &w) > workspace_bytes || !workspace)
    return BFB_ERR_WORKSPACE;
  carve_conv(workspace, dtype, n_in, n_out, K, cin, cout, pair_cap, 1, &w);
  cudaStream_t st = as_stream(stream);
  switch (dtype) {
    case BFB_F32:
      return conv_backward<float>(features, n_in, cin, filters, K, cout, out_bp, n_out, indice_pairs, pair_cap,
                                  indice_num, inverse, input_grad, filters_grad, w, st);
    case BFB_F16:
      return conv_backward<__half>(features, n_in, cin, filters, K, cout, out_bp, n_out, indice_pairs, pair_cap,
                                   indice_num, inverse, input_grad, filters_grad, w, st);
    case BFB_BF16:
      return conv_backward<__nv_bfloat16>(features, n_in, cin, filters, K, cout, out_bp, n_out, indice_pairs,
                                          pair_cap, indice_num, inverse, input_grad, filters_grad, w, st);
    default:
      return BFB_ERR_UNSUPPORTED_DTYPE;
  }
}

extern "C" int bfb_indice_maxpool_workspace_size(int64_t n_in, int64_t n_out, int64_t K, int backward,
                                                 size_t* bytes) {
  if (!bytes || n_in < 0 || n_out < 0 || K <= 0 || K > kMaxK) return BFB_ERR_INVALID_ARG;
  *bytes = align_up(sizeof(int32_t) * (size_t)((backward ? n_in : n_out) * K));
  return BFB_OK;
}

template <class T>
static int maxpool_fwd(const void* f, int64_t C, const int32_t* nbr, int64_t K, int64_t n_out, void* out,
                       cudaStream_t st) {
  if (n_out == 0) return BFB_OK;
  spc_maxpool_kernel<T><<<grid_for(n_out * C, 256), 256, 0, st>>>(static_cast<const T*>(f), (int)C, nbr, (int)K,
                                                                  n_out, static_cast<T*>(out));
  BFB_CHECK_LAUNCH();
  return BFB_OK;
}

template <class T>
static int maxpool_bwd(const void* f, const void* y, const void* gy, int64_t C, const int32_t* nbr, int64_t K,
                       int64_t n_in, void* gx, cudaStream_t st) {
  if (n_in == 0) return BFB_OK;
  spc_maxpool_bwd_kernel<T><<<grid_for(n_in * C, 256), 256, 0, st>>>(
      static_cast<const T*>(f), static_cast<const T*>(y), static_cast<const T*>(gy), (int)C, nbr, (int)K, n_in,
      static_cast<T*>(gx));
  BFB_CHECK_LAUNCH();
  return BFB_OK;
}

extern "C" int bfb_indice_maxpool(const void* features, int dtype, int64_t n_in, int64_t C,
                                  const int32_t* indice_pairs, int64_t K, int64_t pair_cap,
                                  const int32_t* indice_num, int64_t n_out, void* out, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  BFB_INJECT_POINT();
  BFB_TRY(check_conv_args(dtype, n_in, C, K, C, pair_cap, n_out));
  if ((n_in > 0 && !features) || (n_out > 0 && !out) || (pair_cap > 0 && (!indice_pairs || !indice_num)))
    return BFB_ERR_INVALID_ARG;
  if (!workspace || workspace_bytes < sizeof(int32_t) * (size_t)(n_out * K)) return BFB_ERR_WORKSPACE;
  cudaStream_t st = as_stream(stream);
  int32_t* nbr = static_cast<int32_t*>(workspace);
  BFB_TRY(build_tables(indice_pairs, K, pair_cap, indice_num, 0, n_in, n_out, nbr, nullptr, st));
  switch (dtype) {
    case BFB_F32: return maxpool_fwd<float>(features, C, nbr, K, n_out, out, st);
    case BFB_F16: return maxpool_fwd<__half>(features, C, nbr, K, n_out, out, st);
    case BFB_BF16: return maxpool_fwd<__nv_bfloat16>(features, C, nbr, K, n_out, out, st);
    default: return BFB_ERR_UNSUPPORTED_DTYPE;
  }
}

extern "C" int bfb_indice_maxpool_backward(const void* features, const void* out_features, const void* out_bp,
                                           int dtype, int64_t n_in, int64_t n_out, int64_t C,
                                           const int32_t* indice_pairs, int64_t K, int64_t pair_cap,
                                           const int32_t* indice_num, void* input_grad, void* workspace,
                                           size_t workspace_bytes, void* stream) {
  BFB_INJECT_POINT();
  BFB_TRY(check_conv_args(dtype, n_in, C, K, C, pair_cap, n_out));
  if ((n_in > 0 && (!features || !input_grad)) || (n_out > 0 && (!out_features || !out_bp)) ||
      (pair_cap > 0 && (!indice_pairs || !indice_num)))
    return BFB_ERR_INVALID_ARG;
  if (!workspace || workspace_bytes < sizeof(int32_t) * (size_t)(n_in * K)) return BFB_ERR_WORKSPACE;
  cudaStream_t st = as_stream(stream);
  int32_t* nbr = static_cast<int32_t*>(workspace);
  BFB_TRY(build_tables(indice_pairs, K, pair_cap, indice_num, 0, n_in, n_out, nullptr, nbr, st));
  switch (dtype) {
    case BFB_F32: return maxpool_bwd<float>(features, out_features, out_bp, C, nbr, K, n_in, input_grad, st);
    case BFB_F16: return maxpool_bwd<__half>(features, out_features, out_bp, C, nbr, K, n_in, input_grad, st);
    case BFB_BF16:
      return maxpool_bwd<__nv_bfloat16>(features, out_features, out_bp, C, nbr, K, n_in, input_grad, st);
    default: return BFB_ERR_UNSUPPORTED_DTYPE;
  }
}

extern "C" int bfb_spconv_timeouts(uint64_t* count, int reset) { return spconv_timeouts(count, reset); }
