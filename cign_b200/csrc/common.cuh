// Shared device/host helpers for the CIGN sm_100a kernels.
//
// Every entry point of libcign_sm100.so validates its arguments on the host,
// launches on the caller's stream and returns an int status (0 = ok).  The
// message for the last failure on the calling thread is kept in a
// thread-local string readable through cign_last_error().
#pragma once

#include <cuda_runtime.h>
#include <cstdint>
#include <cstddef>

#include "../../include/cign_sm100.h"

namespace cign {

// ---------------------------------------------------------------- errors
int set_error(int code, const char* fmt, ...);
void clear_error();

#define CIGN_REQUIRE(cond, code, ...)                                  \
  do {                                                                  \
    if (!(cond)) return ::cign::set_error((code), __VA_ARGS__);        \
  } while (0)

// Every kernel launch of the library is followed by CIGN_CHECK_LAUNCH, which
// also counts it (cign_kernel_launches()).
void count_launch();

#define CIGN_CHECK_LAUNCH(what)                                               \
  do {                                                                        \
    cudaError_t _e = cudaGetLastError();                                      \
    if (_e != cudaSuccess)                                                    \
      return ::cign::set_error(CIGN_ERR_LAUNCH, "%s: %s", (what),             \
                               cudaGetErrorString(_e));                       \
    ::cign::count_launch();                                                   \
  } while (0)

#define CIGN_CHECK_CUDA(call, what)                                           \
  do {                                                                        \
    cudaError_t _e = (call);                                                  \
    if (_e != cudaSuccess)                                                    \
      return ::cign::set_error(CIGN_ERR_CUDA, "%s: %s", (what),               \
                               cudaGetErrorString(_e));                       \
  } while (0)

inline bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// Number of SMs of the current device (cached per device id).
int sm_count();

// Work split of a CSR-like pointer array: rows with more than `seg_len`
// entries ("heavy" rows, e.g. hubs of a power-law graph) are cut into
// segments of at most seg_len entries, each processed by its own lane
// group; their partial results are combined afterwards in segment order,
// which keeps the sum order fixed (deterministic).  Rows of at most seg_len
// entries are processed whole.  One device buffer holds
//   seg_row[n_seg] | seg_begin[n_seg] | seg_end[n_seg] |
//   heavy_row[n_heavy] | heavy_first[n_heavy + 1] | light_row[n_light]
// (segments of heavy row h are heavy_first[h] .. heavy_first[h+1]-1).
// light_row lists the other rows (at most seg_len entries, empty rows
// included) by length, longest first, ties in row order.  Kernels that
// take whole rows from it give the warps of one CTA rows of (nearly) the
// same length, so a CTA does not hold its SM slot with most of its warps
// finished while one long row completes, and the longest rows start first.
// The order only decides which warp computes a row, not how: every row's
// result is the same as with rows taken in index order.
struct SegList {
  int32_t* buf = nullptr;  // device
  int64_t n_seg = 0;
  int64_t n_heavy = 0;
  int64_t n_light = 0;
  int32_t max_len = 0;
  int32_t seg_len = 0;
  const int32_t* seg_row() const { return buf; }
  const int32_t* seg_begin() const { return buf + n_seg; }
  const int32_t* seg_end() const { return buf + 2 * n_seg; }
  const int32_t* heavy_row() const { return buf + 3 * n_seg; }
  const int32_t* heavy_first() const { return buf + 3 * n_seg + n_heavy; }
  const int32_t* light_row() const { return buf + 3 * n_seg + 2 * n_heavy + 1; }
};

// Reads the device pointer array (int32 [rows+1]) to the host and builds the
// segment list (heavy rows ordered by length, longest first) and the
// length-ordered light-row list.  Plan time only.
int build_segments(const int32_t* ptr_dev, int64_t rows, int seg_len, SegList* out);
void free_segments(SegList* s);

// Deterministic two-stage column sums of a row-major [n, c] matrix
// (reduce.cu).  `partial` holds colsum_chunks(n) * c floats.
int64_t colsum_chunks(int64_t n);
int colsum_f32(const float* a, int64_t n, int64_t c, float* partial,
               float* out, cudaStream_t s);
// out_m[j] = sum over rows r of a_m[r * ld + j] (j < cols) for one or two
// matrices (a1/out1 may be NULL), in a fixed order (reduce.cu).  Used as the
// second stage of the chunked parameter-gradient reductions.
int colsum_rows(const float* a0, float* out0, const float* a1, float* out1, int64_t rows,
                int64_t cols, int64_t ld, cudaStream_t s);

constexpr unsigned kFullMask = 0xffffffffu;

// ---------------------------------------------------------------- math
// SiLU and its derivative written from their definitions:
//   silu(x) = x * sigmoid(x),  silu'(x) = s * (1 + x * (1 - s)).
__device__ __forceinline__ float sigmoid_f(float x) {
  return 1.0f / (1.0f + expf(-x));
}
__device__ __forceinline__ float silu_f(float x) { return x * sigmoid_f(x); }
__device__ __forceinline__ float silu_grad_f(float x) {
  const float s = sigmoid_f(x);
  return s * (1.0f + x * (1.0f - s));
}
__device__ __forceinline__ float leaky_f(float x, float slope) {
  return x > 0.0f ? x : x * slope;
}

// ---------------------------------------------------------------- RNG
// Dropout seed of one call: a value, or (ptr != NULL) the value stored in
// device memory at ptr -- read by the kernel, so a captured CUDA graph can
// draw a new seed on every replay.  Kernels convert it once on entry.
struct Seed {
  uint64_t value = 0;
  const uint64_t* ptr = nullptr;
  Seed() = default;
  Seed(uint64_t v) : value(v) {}  // NOLINT: implicit on purpose (plain seeds)
  Seed(uint64_t v, const uint64_t* p) : value(v), ptr(p) {}
  __device__ __forceinline__ operator uint64_t() const { return ptr != nullptr ? *ptr : value; }
};

// splitmix64 finaliser (Steele, Lea, Flood 2014) -- the counter-based hash
// both dropout streams of the reference use.  idx is hashed as
// seed ^ (idx * 0xD2B74407B1CE6E93).
__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}
__host__ __device__ __forceinline__ uint64_t dropout_hash(uint64_t seed,
                                                          uint64_t idx) {
  return splitmix64(seed ^ (idx * 0xD2B74407B1CE6E93ull));
}
// GAT attention dropout (24-bit-free float uniform from the high 32 bits):
// keep iff ((r >> 32) + 0.5) * 2^-32 > p.   (collapsed_gat_cuda.cu:42-45)
__host__ __device__ __forceinline__ bool gat_keep(uint64_t seed, uint64_t idx,
                                                  float p) {
  const uint32_t hi = static_cast<uint32_t>(dropout_hash(seed, idx) >> 32);
  const float u = (static_cast<float>(hi) + 0.5f) * 2.3283064365386963e-10f;
  return u > p;
}
// Block-op dropout (53-bit double uniform): keep iff (r >> 11) * 2^-53 >= p.
// (fused_block_ops.py:15, dropout_keep)  t = r >> 11 < 2^53, so t * 2^-53 is
// exact in double and so is double(p) * 2^53: the test is the integer
// comparison t >= ceil(double(p) * 2^53), with the threshold loop-invariant.
__host__ __device__ __forceinline__ uint64_t block_keep_threshold(float p) {
  return static_cast<uint64_t>(ceil(static_cast<double>(p) * 9007199254740992.0));
}
__host__ __device__ __forceinline__ bool block_keep(uint64_t seed, uint64_t idx,
                                                    float p) {
  if (p <= 0.0f) return true;
  return (dropout_hash(seed, idx) >> 11) >= block_keep_threshold(p);
}

// ---------------------------------------------------------------- warp
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFullMask, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFullMask, v, o));
  return v;
}

// ---------------------------------------------------------------- cp.async
// 16-byte asynchronous global -> shared copies (LDGSTS, L1 bypass).  Each
// thread waits only for its own groups, so a lane that reads back exactly
// the bytes it copied needs no further synchronisation.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
// The same copy to a shared-memory address given in the shared state space
// (as smem_u32 returns), and the matching 16-byte shared-memory load: with
// explicit state-space addresses the compiler emits LDGSTS / LDS directly.
__device__ __forceinline__ void cp_async16_s(uint32_t saddr, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(saddr), "l"(gmem) : "memory");
}
__device__ __forceinline__ float4 lds_f4(uint32_t saddr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];\n"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(saddr)
               : "memory");
  return v;
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// ---------------------------------------------------------------- TMA ring
// Bulk-copy (TMA, non-tensor) ring of shared-memory slots, one per warp.
// Lane 0 arms a slot's mbarrier with the expected byte count and issues
// cp.async.bulk copies (global -> shared, no multicast) that complete on it;
// all lanes wait for the slot's phase, read it, and the slot is refilled
// after a __syncwarp() and an async-proxy fence.  Waits are bounded: after
// kWaitLimit polls the wait reports failure, the caller records a status
// and drains, so a stuck copy can never hang the GPU.
constexpr unsigned kWaitLimit = 1u << 20;
constexpr int kStatusTimeout = 1;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::
          "r"(dst), "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}
// Bounded wait for `parity` on barrier `bar`; false after kWaitLimit polls.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  for (unsigned i = 0; i < kWaitLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// Persistent-kernel grid: resident CTAs per SM x SMs for `kernel`.
template <typename K>
int persistent_grid(K kernel, int threads, size_t smem) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) !=
          cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  return per_sm * sm_count();
}

// ---------------------------------------------------------------- vectors
template <int VEC> struct VecT;
template <> struct VecT<1> { using type = float; };
template <> struct VecT<4> { using type = float4; };

template <int VEC>
__device__ __forceinline__ typename VecT<VEC>::type ldg_vec(const float* p);
template <>
__device__ __forceinline__ float ldg_vec<1>(const float* p) { return __ldg(p); }
template <>
__device__ __forceinline__ float4 ldg_vec<4>(const float* p) {
  return __ldg(reinterpret_cast<const float4*>(p));
}

template <int VEC>
__device__ __forceinline__ typename VecT<VEC>::type ld_vec(const float* p);
template <>
__device__ __forceinline__ float ld_vec<1>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float4 ld_vec<4>(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}

__device__ __forceinline__ void st_vec(float* p, float v) { *p = v; }
__device__ __forceinline__ void st_vec(float* p, float4 v) {
  *reinterpret_cast<float4*>(p) = v;
}

// Element access on a vector held in registers.
__device__ __forceinline__ float& vel(float& v, int) { return v; }
__device__ __forceinline__ float& vel(float4& v, int i) {
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}
__device__ __forceinline__ float vel(const float& v, int) { return v; }
__device__ __forceinline__ float vel(const float4& v, int i) {
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

__device__ __forceinline__ void vzero(float& v) { v = 0.0f; }
__device__ __forceinline__ void vzero(float4& v) { v = make_float4(0.f, 0.f, 0.f, 0.f); }

// acc += a * x
__device__ __forceinline__ void vfma(float& acc, float a, float x) {
  acc = fmaf(a, x, acc);
}
__device__ __forceinline__ void vfma(float4& acc, float a, const float4& x) {
  acc.x = fmaf(a, x.x, acc.x);
  acc.y = fmaf(a, x.y, acc.y);
  acc.z = fmaf(a, x.z, acc.z);
  acc.w = fmaf(a, x.w, acc.w);
}
__device__ __forceinline__ void vadd(float& acc, float x) { acc += x; }
__device__ __forceinline__ void vadd(float4& acc, const float4& x) {
  acc.x += x.x; acc.y += x.y; acc.z += x.z; acc.w += x.w;
}

// Sum of the vectors p[s * stride], s in [s0, s1), added strictly in s order
// (deterministic); U independent loads are kept in flight.
template <int VEC, int U = 8>
__device__ __forceinline__ typename VecT<VEC>::type ordered_sum(const float* p, int64_t stride,
                                                                int s0, int s1) {
  using V = typename VecT<VEC>::type;
  V acc;
  vzero(acc);
  int s = s0;
  for (; s + U <= s1; s += U) {
    V t[U];
#pragma unroll
    for (int u = 0; u < U; ++u) t[u] = ld_vec<VEC>(p + static_cast<int64_t>(s + u) * stride);
#pragma unroll
    for (int u = 0; u < U; ++u) vadd(acc, t[u]);
  }
  for (; s < s1; ++s) vadd(acc, ld_vec<VEC>(p + static_cast<int64_t>(s) * stride));
  return acc;
}

}  // namespace cign
