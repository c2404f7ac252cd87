// Deterministic column reductions used by the parameter gradients (GAT bias,
// head-mean bias).  Two stages with a fixed summation order: stage 1 sums a
// fixed chunk of rows per (chunk, column) into `partial`, stage 2 sums the
// chunk partials in chunk order.  No atomics, so repeated runs are bitwise
// identical.
#include <algorithm>

#include "common.cuh"

namespace cign {

namespace {

constexpr int kColThreads = 256;

__global__ void colsum_stage1_kernel(const float* __restrict__ a, int64_t n,
                                     int64_t c, int64_t rows_per_chunk,
                                     float* __restrict__ partial) {
  const int64_t chunk = blockIdx.x;
  const int64_t j = static_cast<int64_t>(blockIdx.y) * kColThreads + threadIdx.x;
  if (j >= c) return;
  const int64_t r0 = chunk * rows_per_chunk;
  const int64_t r1 = (r0 + rows_per_chunk < n) ? (r0 + rows_per_chunk) : n;
  float s = 0.0f;
  for (int64_t r = r0; r < r1; ++r) s += a[r * c + j];
  partial[chunk * c + j] = s;
}

__global__ void colsum_stage2_kernel(const float* __restrict__ partial,
                                     int64_t chunks, int64_t c,
                                     float* __restrict__ out) {
  const int64_t j = static_cast<int64_t>(blockIdx.x) * kColThreads + threadIdx.x;
  if (j >= c) return;
  float s = 0.0f;
  for (int64_t k = 0; k < chunks; ++k) s += partial[k * c + j];
  out[j] = s;
}

}  // namespace

// Number of row chunks used for an [n, c] column sum (partial buffer holds
// colsum_chunks(n) * c floats).
int64_t colsum_chunks(int64_t n) { return (n + 127) / 128; }

int colsum_f32(const float* a, int64_t n, int64_t c, float* partial, float* out,
               cudaStream_t s) {
  if (c == 0) return CIGN_OK;
  if (n == 0) {
    CIGN_CHECK_CUDA(cudaMemsetAsync(out, 0, c * sizeof(float), s), "colsum: memset");
    return CIGN_OK;
  }
  const int64_t chunks = colsum_chunks(n);
  const int64_t cblocks = (c + kColThreads - 1) / kColThreads;
  CIGN_REQUIRE(chunks < (1ll << 31) && cblocks < 65536, CIGN_ERR_UNSUPPORTED,
               "colsum: shape too large");
  colsum_stage1_kernel<<<dim3(static_cast<unsigned>(chunks), static_cast<unsigned>(cblocks)),
                         kColThreads, 0, s>>>(a, n, c, 128, partial);
  CIGN_CHECK_LAUNCH("colsum_stage1_kernel");
  colsum_stage2_kernel<<<static_cast<unsigned>(cblocks), kColThreads, 0, s>>>(partial, chunks,
                                                                              c, out);
  CIGN_CHECK_LAUNCH("colsum_stage2_kernel");
  return CIGN_OK;
}

}  // namespace cign
