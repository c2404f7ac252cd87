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
constexpr int kSumWarps = 16;

__global__ void colsum_stage1_kernel(const float* __restrict__ a, int64_t n,
                                     int64_t c, int64_t rows_per_chunk,
                                     float* __restrict__ partial) {
  const int64_t chunk = blockIdx.x;
  const int64_t j = static_cast<int64_t>(blockIdx.y) * kColThreads + threadIdx.x;
  if (j >= c) return;
  const int64_t r0 = chunk * rows_per_chunk;
  const int64_t r1 = (r0 + rows_per_chunk < n) ? (r0 + rows_per_chunk) : n;
  partial[chunk * c + j] = ordered_sum<1>(a + r0 * c + j, c, 0, static_cast<int>(r1 - r0));
}

// out_m[j] = sum over r in [0, rows) of a_m[r * ld + j] for j < cols, for the
// matrix m = blockIdx.y (at most two: a0/out0 and a1/out1).  A block covers
// 32 columns; warp w sums its contiguous share of rows in row order, then the
// warp sums are added in warp order -- a fixed order, so runs are bitwise
// repeatable.
__global__ void __launch_bounds__(kSumWarps * 32)
colsum_rows_kernel(const float* __restrict__ a0, float* __restrict__ out0,
                   const float* __restrict__ a1, float* __restrict__ out1, int rows, int64_t cols,
                   int64_t ld) {
  __shared__ float part[kSumWarps][32];
  const float* a = blockIdx.y == 0 ? a0 : a1;
  float* out = blockIdx.y == 0 ? out0 : out1;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t j = static_cast<int64_t>(blockIdx.x) * 32 + lane;
  const int rpw = (rows + kSumWarps - 1) / kSumWarps;
  const int r0 = w * rpw;
  const int r1 = r0 + rpw < rows ? r0 + rpw : rows;
  float s = 0.0f;
  if (j < cols && r0 < r1) s = ordered_sum<1>(a + j, ld, r0, r1);
  part[w][lane] = s;
  __syncthreads();
  if (w == 0 && j < cols) {
    float t = 0.0f;
#pragma unroll
    for (int k = 0; k < kSumWarps; ++k) t += part[k][lane];
    out[j] = t;
  }
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
  return colsum_rows(partial, out, nullptr, nullptr, chunks, c, c, s);
}

int colsum_rows(const float* a0, float* out0, const float* a1, float* out1, int64_t rows,
                int64_t cols, int64_t ld, cudaStream_t s) {
  if (cols == 0) return CIGN_OK;
  CIGN_REQUIRE(rows > 0 && rows < (1ll << 31), CIGN_ERR_UNSUPPORTED, "colsum: bad row count");
  const int64_t blocks = (cols + 31) / 32;
  CIGN_REQUIRE(blocks < (1ll << 31), CIGN_ERR_UNSUPPORTED, "colsum: too many columns");
  const dim3 grid(static_cast<unsigned>(blocks), a1 != nullptr ? 2u : 1u);
  colsum_rows_kernel<<<grid, kSumWarps * 32, 0, s>>>(a0, out0, a1, out1, static_cast<int>(rows),
                                                      cols, ld);
  CIGN_CHECK_LAUNCH("colsum_rows_kernel");
  return CIGN_OK;
}

}  // namespace cign

using namespace cign;

extern "C" {

size_t cign_colsum_workspace_bytes(int64_t n, int64_t c) {
  if (n <= 0 || c <= 0) return 0;
  return static_cast<size_t>(colsum_chunks(n)) * c * sizeof(float);
}

int cign_colsum_f32(int64_t n, int64_t c, const float* a, float* out, void* ws, size_t ws_bytes,
                    cign_stream_t stream) {
  CIGN_REQUIRE(n >= 0 && c >= 0, CIGN_ERR_INVALID_ARGUMENT, "colsum: negative size");
  if (c == 0) return CIGN_OK;
  CIGN_REQUIRE(out != nullptr && (n == 0 || a != nullptr), CIGN_ERR_NULL_POINTER,
               "colsum: NULL argument");
  const size_t need = cign_colsum_workspace_bytes(n, c);
  CIGN_REQUIRE(ws_bytes >= need && (need == 0 || ws != nullptr), CIGN_ERR_INVALID_ARGUMENT,
               "colsum: workspace too small (%zu < %zu bytes)", ws_bytes, need);
  return colsum_f32(a, n, c, static_cast<float*>(ws), out, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
