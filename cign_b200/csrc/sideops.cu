// GAT side ops: attention logits (alpha_src/alpha_dst) with their backward,
// and the head-mean + bias + SiLU epilogue used by the non-collapsed path.
//
// Reference: fused_gat_sideops_ext/fused_gat_sideops_cuda.cu (attention
// forward :25-60, backward :65-167, head-SiLU :171-239) behind
// fused_gat_sideops.py:50-105.
//
// The logits backward is one pass over x: every CTA owns a chunk of nodes
// and a 1024-float column tile of x's [H*C] row, writes grad_x for it and
// accumulates the att_src/att_dst parameter gradients of that chunk in
// registers; a second tiny kernel adds the chunk partials in chunk order.
#include <algorithm>

#include "common.cuh"

namespace cign {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxChunks = 512;

template <int VEC>
__global__ void __launch_bounds__(kThreads)
attn_logits_fwd_kernel(int64_t NH, int H, int64_t C, const float* __restrict__ x,
                       const float* __restrict__ att_src,
                       const float* __restrict__ att_dst,
                       float* __restrict__ alpha_src, float* __restrict__ alpha_dst) {
  using V = typename VecT<VEC>::type;
  const int64_t nh = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (nh >= NH) return;
  const int h = static_cast<int>(nh % H);
  const float* xr = x + nh * C;
  const float* as = att_src + static_cast<int64_t>(h) * C;
  const float* ad = att_dst + static_cast<int64_t>(h) * C;
  float ss = 0.0f, sd = 0.0f;
  for (int64_t c = static_cast<int64_t>(lane) * VEC; c < C; c += 32 * VEC) {
    const V xv = ldg_vec<VEC>(xr + c);
    const V av = ldg_vec<VEC>(as + c);
    const V dv = ldg_vec<VEC>(ad + c);
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      ss = fmaf(vel(xv, j), vel(av, j), ss);
      sd = fmaf(vel(xv, j), vel(dv, j), sd);
    }
  }
  ss = warp_sum(ss);
  sd = warp_sum(sd);
  if (lane == 0) {
    alpha_src[nh] = ss;
    alpha_dst[nh] = sd;
  }
}

// grid = (chunks, column tiles of kThreads*VEC floats over H*C)
template <int VEC>
__global__ void __launch_bounds__(kThreads)
attn_logits_bwd_kernel(int64_t n, int H, int64_t C, int64_t rows_per_chunk,
                       const float* __restrict__ gsrc, const float* __restrict__ gdst,
                       const float* __restrict__ x, const float* __restrict__ att_src,
                       const float* __restrict__ att_dst, float* __restrict__ grad_x,
                       int accumulate, float* __restrict__ partial) {
  using V = typename VecT<VEC>::type;
  const int64_t HC = static_cast<int64_t>(H) * C;
  const int64_t chunk = blockIdx.x;
  const int64_t col = (static_cast<int64_t>(blockIdx.y) * kThreads + threadIdx.x) * VEC;
  if (col >= HC) return;
  const int h = static_cast<int>(col / C);
  const V as = ldg_vec<VEC>(att_src + col);
  const V ad = ldg_vec<VEC>(att_dst + col);
  V ps, pd;
  vzero(ps);
  vzero(pd);
  const int64_t r0 = chunk * rows_per_chunk;
  const int64_t r1 = (r0 + rows_per_chunk < n) ? (r0 + rows_per_chunk) : n;
  for (int64_t r = r0; r < r1; ++r) {
    const float gs = __ldg(gsrc + r * H + h);
    const float gd = __ldg(gdst + r * H + h);
    const V xv = ldg_vec<VEC>(x + r * HC + col);
    V gx;
    if (accumulate) gx = ld_vec<VEC>(grad_x + r * HC + col);
    else vzero(gx);
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      vel(gx, j) += gs * vel(as, j) + gd * vel(ad, j);
      vel(ps, j) = fmaf(gs, vel(xv, j), vel(ps, j));
      vel(pd, j) = fmaf(gd, vel(xv, j), vel(pd, j));
    }
    st_vec(grad_x + r * HC + col, gx);
  }
  st_vec(partial + (chunk * 2 + 0) * HC + col, ps);
  st_vec(partial + (chunk * 2 + 1) * HC + col, pd);
}

__global__ void head_silu_fwd_kernel(int64_t n, int H, int64_t C,
                                     const float* __restrict__ out,
                                     const float* __restrict__ bias,
                                     float* __restrict__ y, float* __restrict__ pre) {
  const int64_t total = n * C;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const float hf = static_cast<float>(H);
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += stride) {
    const int64_t r = i / C, c = i - r * C;
    const float* o = out + r * H * C + c;
    float s = 0.0f;
    for (int h = 0; h < H; ++h) s += o[static_cast<int64_t>(h) * C];
    const float p = s / hf + bias[c];
    pre[i] = p;
    y[i] = silu_f(p);
  }
}

__global__ void head_silu_bwd_kernel(int64_t n, int H, int64_t C,
                                     const float* __restrict__ gy,
                                     const float* __restrict__ pre,
                                     float* __restrict__ grad_out,
                                     float* __restrict__ gpre) {
  const int64_t total = n * C;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const float hf = static_cast<float>(H);
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += stride) {
    const int64_t r = i / C, c = i - r * C;
    const float gp = gy[i] * silu_grad_f(pre[i]);
    if (gpre != nullptr) gpre[i] = gp;
    const float g = gp / hf;
    float* go = grad_out + r * H * C + c;
    for (int h = 0; h < H; ++h) go[static_cast<int64_t>(h) * C] = g;
  }
}

int64_t attn_rows_per_chunk(int64_t n) {
  return std::max<int64_t>(64, (n + kMaxChunks - 1) / kMaxChunks);
}

int grid_1d(int64_t total) {
  const int64_t want = (total + kThreads - 1) / kThreads;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, 148ll * 16)));
}

}  // namespace
}  // namespace cign

using namespace cign;

extern "C" {

int cign_attn_logits_fwd(int64_t n, int32_t heads, int32_t channels, const float* x,
                         const float* att_src, const float* att_dst, float* alpha_src,
                         float* alpha_dst, cign_stream_t stream) {
  CIGN_REQUIRE(n >= 0 && heads >= 1 && channels >= 1, CIGN_ERR_INVALID_ARGUMENT,
               "attn_logits_fwd: bad sizes");
  if (n == 0) return CIGN_OK;
  CIGN_REQUIRE(x && att_src && att_dst && alpha_src && alpha_dst, CIGN_ERR_NULL_POINTER,
               "attn_logits_fwd: NULL argument");
  const int64_t NH = n * heads;
  const int64_t blocks = (NH * 32 + kThreads - 1) / kThreads;
  CIGN_REQUIRE(blocks < (1ll << 31), CIGN_ERR_UNSUPPORTED, "attn_logits_fwd: too large");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool v4 = channels % 4 == 0 && aligned16(x) && aligned16(att_src) && aligned16(att_dst);
  if (v4)
    attn_logits_fwd_kernel<4><<<static_cast<unsigned>(blocks), kThreads, 0, s>>>(
        NH, heads, channels, x, att_src, att_dst, alpha_src, alpha_dst);
  else
    attn_logits_fwd_kernel<1><<<static_cast<unsigned>(blocks), kThreads, 0, s>>>(
        NH, heads, channels, x, att_src, att_dst, alpha_src, alpha_dst);
  CIGN_CHECK_LAUNCH("attn_logits_fwd_kernel");
  return CIGN_OK;
}

size_t cign_attn_logits_bwd_workspace_bytes(int64_t n, int32_t heads, int32_t channels) {
  if (n <= 0) return 0;
  const int64_t chunks = (n + attn_rows_per_chunk(n) - 1) / attn_rows_per_chunk(n);
  return static_cast<size_t>(chunks) * 2 * heads * channels * sizeof(float);
}

int cign_attn_logits_bwd(int64_t n, int32_t heads, int32_t channels, const float* grad_src,
                         const float* grad_dst, const float* x, const float* att_src,
                         const float* att_dst, float* grad_x, float* grad_att_src,
                         float* grad_att_dst, int32_t accumulate, void* ws,
                         size_t ws_bytes, cign_stream_t stream) {
  CIGN_REQUIRE(n >= 0 && heads >= 1 && channels >= 1, CIGN_ERR_INVALID_ARGUMENT,
               "attn_logits_bwd: bad sizes");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t HC = static_cast<int64_t>(heads) * channels;
  CIGN_REQUIRE(grad_att_src && grad_att_dst, CIGN_ERR_NULL_POINTER,
               "attn_logits_bwd: NULL parameter gradient");
  if (n == 0) {
    CIGN_CHECK_CUDA(cudaMemsetAsync(grad_att_src, 0, HC * sizeof(float), s), "memset");
    CIGN_CHECK_CUDA(cudaMemsetAsync(grad_att_dst, 0, HC * sizeof(float), s), "memset");
    return CIGN_OK;
  }
  CIGN_REQUIRE(grad_src && grad_dst && x && att_src && att_dst && grad_x, CIGN_ERR_NULL_POINTER,
               "attn_logits_bwd: NULL argument");
  const size_t need = cign_attn_logits_bwd_workspace_bytes(n, heads, channels);
  CIGN_REQUIRE(ws != nullptr && ws_bytes >= need, CIGN_ERR_INVALID_ARGUMENT,
               "attn_logits_bwd: workspace too small (%zu < %zu)", ws_bytes, need);
  const int64_t rpc = attn_rows_per_chunk(n);
  const int64_t chunks = (n + rpc - 1) / rpc;
  const bool v4 = channels % 4 == 0 && aligned16(x) && aligned16(att_src) &&
                  aligned16(att_dst) && aligned16(grad_x) && aligned16(ws);
  const int vec = v4 ? 4 : 1;
  const int64_t tiles = (HC / vec + kThreads - 1) / kThreads;
  CIGN_REQUIRE(tiles < 65536, CIGN_ERR_UNSUPPORTED, "attn_logits_bwd: H*C too large");
  float* partial = static_cast<float*>(ws);
  dim3 grid(static_cast<unsigned>(chunks), static_cast<unsigned>(tiles));
  if (v4)
    attn_logits_bwd_kernel<4><<<grid, kThreads, 0, s>>>(n, heads, channels, rpc, grad_src,
                                                        grad_dst, x, att_src, att_dst, grad_x,
                                                        accumulate, partial);
  else
    attn_logits_bwd_kernel<1><<<grid, kThreads, 0, s>>>(n, heads, channels, rpc, grad_src,
                                                        grad_dst, x, att_src, att_dst, grad_x,
                                                        accumulate, partial);
  CIGN_CHECK_LAUNCH("attn_logits_bwd_kernel");
  // partial rows alternate src, dst per chunk: two [chunks, HC] matrices with ld 2*HC
  return colsum_rows(partial, grad_att_src, partial + HC, grad_att_dst, chunks, HC, 2 * HC, s);
}

int cign_head_mean_bias_silu_fwd(int64_t n, int32_t heads, int32_t channels,
                                 const float* out, const float* bias, float* y, float* pre,
                                 cign_stream_t stream) {
  CIGN_REQUIRE(n >= 0 && heads >= 1 && channels >= 1, CIGN_ERR_INVALID_ARGUMENT,
               "head_mean_bias_silu_fwd: bad sizes");
  if (n == 0) return CIGN_OK;
  CIGN_REQUIRE(out && bias && y && pre, CIGN_ERR_NULL_POINTER,
               "head_mean_bias_silu_fwd: NULL argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  head_silu_fwd_kernel<<<grid_1d(n * channels), kThreads, 0, s>>>(n, heads, channels, out, bias,
                                                                  y, pre);
  CIGN_CHECK_LAUNCH("head_silu_fwd_kernel");
  return CIGN_OK;
}

size_t cign_head_mean_bias_silu_bwd_workspace_bytes(int64_t n, int32_t channels) {
  auto r = [](size_t b) { return (b + 255) / 256 * 256; };
  return r(static_cast<size_t>(n) * channels * sizeof(float)) +
         r(static_cast<size_t>(colsum_chunks(n)) * channels * sizeof(float));
}

int cign_head_mean_bias_silu_bwd(int64_t n, int32_t heads, int32_t channels,
                                 const float* grad_y, const float* pre, float* grad_out,
                                 float* grad_bias, void* ws, size_t ws_bytes,
                                 cign_stream_t stream) {
  CIGN_REQUIRE(n >= 0 && heads >= 1 && channels >= 1, CIGN_ERR_INVALID_ARGUMENT,
               "head_mean_bias_silu_bwd: bad sizes");
  CIGN_REQUIRE(grad_bias != nullptr, CIGN_ERR_NULL_POINTER, "head_mean_bias_silu_bwd: grad_bias");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n == 0) {
    CIGN_CHECK_CUDA(cudaMemsetAsync(grad_bias, 0, channels * sizeof(float), s), "memset");
    return CIGN_OK;
  }
  CIGN_REQUIRE(grad_y && pre && grad_out, CIGN_ERR_NULL_POINTER,
               "head_mean_bias_silu_bwd: NULL argument");
  const size_t need = cign_head_mean_bias_silu_bwd_workspace_bytes(n, channels);
  CIGN_REQUIRE(ws != nullptr && ws_bytes >= need, CIGN_ERR_INVALID_ARGUMENT,
               "head_mean_bias_silu_bwd: workspace too small");
  float* gpre = static_cast<float*>(ws);
  float* partial = reinterpret_cast<float*>(
      static_cast<char*>(ws) + (static_cast<size_t>(n) * channels * sizeof(float) + 255) / 256 * 256);
  // one head: grad_out is g_pre itself, so the column sums read it directly
  head_silu_bwd_kernel<<<grid_1d(n * channels), kThreads, 0, s>>>(
      n, heads, channels, grad_y, pre, grad_out, heads == 1 ? nullptr : gpre);
  CIGN_CHECK_LAUNCH("head_silu_bwd_kernel");
  return colsum_f32(heads == 1 ? grad_out : gpre, n, channels, partial, grad_bias, s);
}

}  // extern "C"
