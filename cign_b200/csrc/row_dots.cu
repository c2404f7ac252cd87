// Row dots: out[n, k] = <x[n, :], V[k, :]> for a small number K of vectors,
// and the backward pair grad_x += g V, grad_V = g^T x.
//
// The aggregate-first GAT uses it for its attention logits
// (fused_gat_sideops.py:50-71 on lin(x).view(N, H, C), generic_engine/
// model_cign.py:551-567): with lin.weight = W [H*C, D],
//   alpha_src[n, h] = <W_h x_n, att_src[h]> = <x_n, W_h^T att_src[h]>,
// so the 2H logits of a node are K = 2H dots of its D-float row with
// V = [W_h^T att_src[h] ; W_h^T att_dst[h]] -- one read of x, no [N, H*C]
// tensor.  Everything is fp32 with a fixed summation order.
//
// Forward: one warp per row; lane l owns columns 4l + 128i, the K partial
// dots are reduced across the warp (same order as the hop gate).
// Backward: grid (row chunks, 128-float column tiles), one float4 of
// columns per lane; per row grad_x = (existing) + sum_k g[n,k] V[k,:] is
// written, and g[n,k] x[n,:] accumulates per lane into K float4 partials
// that the block sums in warp order into [chunks, K, D]; a fixed-order
// column sum over the chunks gives grad_V.
#include <algorithm>

#include "common.cuh"

namespace cign {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxK = 16;
constexpr int kTileCols = 128;

template <int K>
__global__ void __launch_bounds__(kThreads)
row_dots_fwd_kernel(int64_t n, int64_t D, const float* __restrict__ x,
                    const float* __restrict__ V, float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (kThreads / 32) + (threadIdx.x >> 5);
  if (row >= n) return;
  float dot[K];
#pragma unroll
  for (int k = 0; k < K; ++k) dot[k] = 0.0f;
  for (int64_t c = static_cast<int64_t>(lane) * 4; c < D; c += 128) {
    const float4 xv = ld_vec<4>(x + row * D + c);
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const float4 v = ldg_vec<4>(V + k * D + c);
      float t = dot[k];
      t = fmaf(xv.x, v.x, t); t = fmaf(xv.y, v.y, t); t = fmaf(xv.z, v.z, t); t = fmaf(xv.w, v.w, t);
      dot[k] = t;
    }
  }
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const float s = warp_sum(dot[k]);
    if (lane == k) out[row * K + k] = s;
  }
}

template <int K>
__global__ void __launch_bounds__(kThreads)
row_dots_bwd_kernel(int64_t n, int64_t D, int64_t rpc, const float* __restrict__ x,
                    const float* __restrict__ V, const float* __restrict__ g,
                    float* __restrict__ gx, int accumulate, float* __restrict__ pv) {
  __shared__ float4 red[kThreads / 32][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t c = static_cast<int64_t>(blockIdx.y) * kTileCols + lane * 4;
  const bool cv = c < D;
  float4 v[K], a[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    v[k] = cv ? ldg_vec<4>(V + k * D + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    a[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rpc;
  const int64_t r1 = r0 + rpc < n ? r0 + rpc : n;
  if (cv) {
    // kRowBatch rows per pass with all their loads issued first: the rows
    // a warp walks are independent, so their latencies overlap; partials
    // still accumulate row by row in increasing order.
    constexpr int kRowBatch = 4;
    constexpr int64_t kStride = kThreads / 32;
    for (int64_t base = r0 + warp; base < r1; base += kRowBatch * kStride) {
      float4 xv[kRowBatch], t[kRowBatch];
#pragma unroll
      for (int b = 0; b < kRowBatch; ++b) {
        const int64_t row = base + b * kStride;
        if (row < r1) {
          xv[b] = ld_vec<4>(x + row * D + c);
          t[b] = accumulate ? ld_vec<4>(gx + row * D + c) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
#pragma unroll
      for (int b = 0; b < kRowBatch; ++b) {
        const int64_t row = base + b * kStride;
        if (row >= r1) break;
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int k = 0; k < K; ++k) {
          const float gk = __ldg(g + row * K + k);
          vfma(o, gk, v[k]);
          vfma(a[k], gk, xv[b]);
        }
        // existing gradient first, then this op's part
        vadd(t[b], o);
        st_vec(gx + row * D + c, t[b]);
      }
    }
  }
  // fixed-order sum of the warps' partials, one k at a time
#pragma unroll
  for (int k = 0; k < K; ++k) {
    red[warp][lane] = a[k];
    __syncthreads();
    if (threadIdx.x < 32) {
      float4 acc = red[0][threadIdx.x];
      for (int w = 1; w < kThreads / 32; ++w) vadd(acc, red[w][threadIdx.x]);
      const int64_t cc = static_cast<int64_t>(blockIdx.y) * kTileCols + threadIdx.x * 4;
      if (cc < D) st_vec(pv + (static_cast<int64_t>(blockIdx.x) * K + k) * D + cc, acc);
    }
    __syncthreads();
  }
}

int64_t rd_rows_per_chunk(int64_t n) {
  const int64_t want = (n + 2 * 148 - 1) / (2 * 148);
  return std::max<int64_t>(64, (want + 7) / 8 * 8);
}
int64_t rd_chunks(int64_t n) { return (n + rd_rows_per_chunk(n) - 1) / rd_rows_per_chunk(n); }

int check_rd(int64_t n, int64_t d, int32_t k, const void* x, const void* V, const char* name) {
  CIGN_REQUIRE(n >= 0 && d >= 1 && k >= 1 && k <= kMaxK, CIGN_ERR_INVALID_ARGUMENT,
               "%s: need n >= 0, d >= 1, 1 <= k <= %d", name, kMaxK);
  CIGN_REQUIRE(d % 4 == 0, CIGN_ERR_UNSUPPORTED, "%s: d must be a multiple of 4", name);
  if (n == 0) return CIGN_OK;
  CIGN_REQUIRE(x != nullptr && V != nullptr, CIGN_ERR_NULL_POINTER, "%s: NULL argument", name);
  CIGN_REQUIRE(aligned16(x) && aligned16(V), CIGN_ERR_ALIGNMENT,
               "%s: x and V must be 16-byte aligned", name);
  return CIGN_OK;
}

#define CIGN_RD_K_DISPATCH(k, CALL)                                                     \
  switch (k) {                                                                          \
    case 1: { constexpr int K_ = 1; CALL; break; }                                      \
    case 2: { constexpr int K_ = 2; CALL; break; }                                      \
    case 3: { constexpr int K_ = 3; CALL; break; }                                      \
    case 4: { constexpr int K_ = 4; CALL; break; }                                      \
    case 5: { constexpr int K_ = 5; CALL; break; }                                      \
    case 6: { constexpr int K_ = 6; CALL; break; }                                      \
    case 7: { constexpr int K_ = 7; CALL; break; }                                      \
    case 8: { constexpr int K_ = 8; CALL; break; }                                      \
    case 9: { constexpr int K_ = 9; CALL; break; }                                      \
    case 10: { constexpr int K_ = 10; CALL; break; }                                    \
    case 11: { constexpr int K_ = 11; CALL; break; }                                    \
    case 12: { constexpr int K_ = 12; CALL; break; }                                    \
    case 13: { constexpr int K_ = 13; CALL; break; }                                    \
    case 14: { constexpr int K_ = 14; CALL; break; }                                    \
    case 15: { constexpr int K_ = 15; CALL; break; }                                    \
    default: { constexpr int K_ = 16; CALL; break; }                                    \
  }

}  // namespace
}  // namespace cign

using namespace cign;

extern "C" {

int cign_row_dots_fwd(int64_t n, int64_t d, int32_t k, const float* x, const float* V,
                      float* out, cign_stream_t stream) {
  int rc = check_rd(n, d, k, x, V, "row_dots_fwd");
  if (rc) return rc;
  if (n == 0) return CIGN_OK;
  CIGN_REQUIRE(out != nullptr, CIGN_ERR_NULL_POINTER, "row_dots_fwd: NULL output");
  const int64_t blocks = (n + kThreads / 32 - 1) / (kThreads / 32);
  CIGN_REQUIRE(blocks < (1ll << 31), CIGN_ERR_UNSUPPORTED, "row_dots_fwd: too many rows");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CIGN_RD_K_DISPATCH(k, (row_dots_fwd_kernel<K_><<<static_cast<unsigned>(blocks), kThreads, 0, s>>>(
                            n, d, x, V, out)));
  CIGN_CHECK_LAUNCH("row_dots_fwd_kernel");
  return CIGN_OK;
}

size_t cign_row_dots_bwd_workspace_bytes(int64_t n, int64_t d, int32_t k) {
  if (n <= 0 || d <= 0 || k <= 0) return 0;
  return static_cast<size_t>(rd_chunks(n)) * k * d * sizeof(float);
}

int cign_row_dots_bwd(int64_t n, int64_t d, int32_t k, const float* x, const float* V,
                      const float* grad_out, float* grad_x, int32_t accumulate, float* grad_V,
                      void* ws, size_t ws_bytes, cign_stream_t stream) {
  int rc = check_rd(n, d, k, x, V, "row_dots_bwd");
  if (rc) return rc;
  CIGN_REQUIRE(grad_V != nullptr, CIGN_ERR_NULL_POINTER, "row_dots_bwd: NULL grad_V");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n == 0) {
    CIGN_CHECK_CUDA(cudaMemsetAsync(grad_V, 0, static_cast<size_t>(k) * d * sizeof(float), s),
                    "row_dots_bwd: memset");
    return CIGN_OK;
  }
  CIGN_REQUIRE(grad_out != nullptr && grad_x != nullptr && ws != nullptr, CIGN_ERR_NULL_POINTER,
               "row_dots_bwd: NULL argument");
  CIGN_REQUIRE(aligned16(grad_x), CIGN_ERR_ALIGNMENT, "row_dots_bwd: grad_x must be 16-byte aligned");
  const size_t need = cign_row_dots_bwd_workspace_bytes(n, d, k);
  CIGN_REQUIRE(ws_bytes >= need, CIGN_ERR_INVALID_ARGUMENT,
               "row_dots_bwd: workspace too small (%zu < %zu bytes)", ws_bytes, need);
  const int64_t rpc = rd_rows_per_chunk(n), ch = rd_chunks(n);
  const int64_t tiles = (d + kTileCols - 1) / kTileCols;
  CIGN_REQUIRE(ch < (1ll << 31) && tiles < 65536, CIGN_ERR_UNSUPPORTED, "row_dots_bwd: too large");
  float* pv = static_cast<float*>(ws);
  const dim3 grid(static_cast<unsigned>(ch), static_cast<unsigned>(tiles));
  CIGN_RD_K_DISPATCH(k, (row_dots_bwd_kernel<K_><<<grid, kThreads, 0, s>>>(
                            n, d, rpc, x, V, grad_out, grad_x, accumulate, pv)));
  CIGN_CHECK_LAUNCH("row_dots_bwd_kernel");
  return colsum_rows(pv, grad_V, nullptr, nullptr, ch, static_cast<int64_t>(k) * d,
                     static_cast<int64_t>(k) * d, s);
}

}  // extern "C"
