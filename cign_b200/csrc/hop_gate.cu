// Hop gate of the CIGN block (generic_engine/model_cign.py:721-749):
//   gate_input = [H + C | |H - C|]   (score mode "new")  or  [H | C]  ("old")
//   alpha      = softmax_k(gate_input @ W^T + b),   W [K, 2D], b [K]
// evaluated without materialising gate_input, the [N, K] logits or the
// softmax, and with the K-wide linear in fp32 (the reference keeps the hop
// gate in fp32, :746).
//
// Forward: one warp per node; each lane forms its float4 slices of the two
// gate halves, dots them with W's rows (read through the read-only cache),
// the K partial dots are reduced across the warp and the softmax is taken.
// Backward: grid (row chunks, 128-float column tiles).  Per node the
// softmax backward g_logit = alpha * (g_alpha - <alpha, g_alpha>) is formed
// by every lane, then per column
//   g_in = sum_k g_logit[k] W[k, :],  dH/dC from g_in through the +, -, |.|
// (d|x|/dx = sign(x), 0 at 0, as torch's abs backward), and the W / b
// gradients accumulate per block (fixed order) into chunk partials that a
// fixed-order column sum reduces.
#include <algorithm>
#include <initializer_list>

#include "common.cuh"

namespace cign {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxK = 8;
constexpr int kTileCols = 128;  // columns of D per backward block (one float4 per lane)

__device__ __forceinline__ float sign_f(float x) { return x > 0.0f ? 1.0f : (x < 0.0f ? -1.0f : 0.0f); }

template <int K>
__global__ void __launch_bounds__(kThreads)
hop_gate_fwd_kernel(int64_t n, int64_t D, int mode, const float* __restrict__ H,
                    const float* __restrict__ C, const float* __restrict__ W,
                    const float* __restrict__ b, float* __restrict__ alpha) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (kThreads / 32) + (threadIdx.x >> 5);
  if (row >= n) return;
  const int64_t D2 = 2 * D;
  float dot[K];
#pragma unroll
  for (int k = 0; k < K; ++k) dot[k] = 0.0f;
  for (int64_t c = static_cast<int64_t>(lane) * 4; c < D; c += 128) {
    const float4 h = ld_vec<4>(H + row * D + c);
    const float4 x = ld_vec<4>(C + row * D + c);
    float4 g0, g1;
    if (mode == 1) {
      g0 = make_float4(h.x + x.x, h.y + x.y, h.z + x.z, h.w + x.w);
      g1 = make_float4(fabsf(h.x - x.x), fabsf(h.y - x.y), fabsf(h.z - x.z), fabsf(h.w - x.w));
    } else {
      g0 = h;
      g1 = x;
    }
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const float4 w0 = ldg_vec<4>(W + k * D2 + c);
      const float4 w1 = ldg_vec<4>(W + k * D2 + D + c);
      float d = dot[k];
      d = fmaf(g0.x, w0.x, d); d = fmaf(g0.y, w0.y, d); d = fmaf(g0.z, w0.z, d); d = fmaf(g0.w, w0.w, d);
      d = fmaf(g1.x, w1.x, d); d = fmaf(g1.y, w1.y, d); d = fmaf(g1.z, w1.z, d); d = fmaf(g1.w, w1.w, d);
      dot[k] = d;
    }
  }
  float m = -INFINITY;
#pragma unroll
  for (int k = 0; k < K; ++k) {
    dot[k] = warp_sum(dot[k]) + __ldg(b + k);
    m = fmaxf(m, dot[k]);
  }
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < K; ++k) {
    dot[k] = expf(dot[k] - m);
    s += dot[k];
  }
  if (lane < K) {
    float v = 0.0f;
#pragma unroll
    for (int k = 0; k < K; ++k)
      if (k == lane) v = dot[k];
    alpha[row * K + lane] = v / s;
  }
}

// grid (chunks, column tiles); rows [chunk*rpc, ...) strided over the warps.
// partial layout: pw [chunks, K, 2D] (this tile's columns), pb [chunks, K]
// (tile 0 only).
template <int K>
// two CTAs per SM (<= 128 registers) up to K = 3 hops; more hops keep their
// per-lane partials in registers at one CTA per SM instead of spilling
__global__ void __launch_bounds__(kThreads, K <= 3 ? 2 : 1)
hop_gate_bwd_kernel(int64_t n, int64_t D, int64_t rpc, int mode, const float* __restrict__ H,
                    const float* __restrict__ C, const float* __restrict__ W,
                    const float* __restrict__ alpha, const float* __restrict__ g_alpha,
                    float* __restrict__ gH, float* __restrict__ gC, int accumulate,
                    const float* __restrict__ add_h, const float* __restrict__ add_c,
                    int64_t add_ld, float* __restrict__ pw, float* __restrict__ pb) {
  __shared__ float4 red[kThreads / 32][2][32];
  __shared__ float redb[kThreads / 32][K];
  __shared__ float4 wt[2][K][32];  // this tile's columns of W's two halves
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t c = static_cast<int64_t>(blockIdx.y) * kTileCols + lane * 4;
  const bool cv = c < D;
  const int64_t D2 = 2 * D;
  float4 a0[K], a1[K];
  float ab[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    a0[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    a1[k] = a0[k];
    ab[k] = 0.0f;
  }
  for (int i = threadIdx.x; i < 2 * K * 32; i += kThreads) {
    const int half = i / (K * 32), k = (i / 32) % K, l = i % 32;
    const int64_t cc = static_cast<int64_t>(blockIdx.y) * kTileCols + l * 4;
    wt[half][k][l] = cc < D ? ldg_vec<4>(W + k * D2 + half * D + cc)
                            : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __syncthreads();
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rpc;
  const int64_t r1 = r0 + rpc < n ? r0 + rpc : n;
  // Two of the warp's rows per iteration (row, then row + kThreads/32: the
  // order of the single-row loop), with both rows' loads issued before
  // either is used, so twice the bytes are in flight per warp.
  struct RowIn {
    float al[K], ga[K];
    float4 h, x, th, tc;
  };
  auto load = [&](int64_t row, RowIn& in) {
#pragma unroll
    for (int k = 0; k < K; ++k) {
      in.al[k] = __ldg(alpha + row * K + k);
      in.ga[k] = __ldg(g_alpha + row * K + k);
    }
    if (!cv) return;
    in.h = ld_vec<4>(H + row * D + c);
    in.x = ld_vec<4>(C + row * D + c);
    // existing gradient first, then the extra addend, then this op's part
    in.th = make_float4(0.f, 0.f, 0.f, 0.f);
    in.tc = in.th;
    if (accumulate) {
      in.th = ld_vec<4>(gH + row * D + c);
      in.tc = ld_vec<4>(gC + row * D + c);
    }
    if (add_h != nullptr) vadd(in.th, ld_vec<4>(add_h + row * add_ld + c));
    if (add_c != nullptr) vadd(in.tc, ld_vec<4>(add_c + row * add_ld + c));
  };
  auto apply = [&](int64_t row, RowIn& in) {
    float gl[K];
    float dotp = 0.0f;
#pragma unroll
    for (int k = 0; k < K; ++k) dotp = fmaf(in.al[k], in.ga[k], dotp);
#pragma unroll
    for (int k = 0; k < K; ++k) {
      gl[k] = in.al[k] * (in.ga[k] - dotp);
      ab[k] += gl[k];
    }
    if (!cv) return;
    const float4 h = in.h, x = in.x;
    float4 s0, s1;
    if (mode == 1) {
      s0 = make_float4(h.x + x.x, h.y + x.y, h.z + x.z, h.w + x.w);
      s1 = make_float4(fabsf(h.x - x.x), fabsf(h.y - x.y), fabsf(h.z - x.z), fabsf(h.w - x.w));
    } else {
      s0 = h;
      s1 = x;
    }
    float4 gi0 = make_float4(0.f, 0.f, 0.f, 0.f), gi1 = gi0;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      vfma(gi0, gl[k], wt[0][k][lane]);
      vfma(gi1, gl[k], wt[1][k][lane]);
      vfma(a0[k], gl[k], s0);
      vfma(a1[k], gl[k], s1);
    }
    float4 oh, oc;
    if (mode == 1) {
      const float sx = sign_f(h.x - x.x), sy = sign_f(h.y - x.y), sz = sign_f(h.z - x.z),
                  sw = sign_f(h.w - x.w);
      oh = make_float4(gi0.x + sx * gi1.x, gi0.y + sy * gi1.y, gi0.z + sz * gi1.z, gi0.w + sw * gi1.w);
      oc = make_float4(gi0.x - sx * gi1.x, gi0.y - sy * gi1.y, gi0.z - sz * gi1.z, gi0.w - sw * gi1.w);
    } else {
      oh = gi0;
      oc = gi1;
    }
    vadd(in.th, oh);
    vadd(in.tc, oc);
    st_vec(gH + row * D + c, in.th);
    st_vec(gC + row * D + c, in.tc);
  };
  constexpr int kW = kThreads / 32;
  for (int64_t row = r0 + warp; row < r1; row += 2 * kW) {
    const bool two = row + kW < r1;
    RowIn a, b;
    load(row, a);
    if (two) load(row + kW, b);
    apply(row, a);
    if (two) apply(row + kW, b);
  }
  // fixed-order reduction of the warps' parameter partials, one k at a time
#pragma unroll
  for (int k = 0; k < K; ++k) {
    red[warp][0][lane] = a0[k];
    red[warp][1][lane] = a1[k];
    if (lane == 0) redb[warp][k] = ab[k];
    __syncthreads();
    if (threadIdx.x < 64) {
      const int l = threadIdx.x & 31, half = threadIdx.x >> 5;
      float4 acc = red[0][half][l];
      for (int w = 1; w < kThreads / 32; ++w) vadd(acc, red[w][half][l]);
      const int64_t cc = static_cast<int64_t>(blockIdx.y) * kTileCols + l * 4;
      if (cc < D) st_vec(pw + (static_cast<int64_t>(blockIdx.x) * K + k) * D2 + half * D + cc, acc);
    }
    __syncthreads();
  }
  if (blockIdx.y == 0 && threadIdx.x < K) {
    float acc = redb[0][threadIdx.x];
    for (int w = 1; w < kThreads / 32; ++w) acc += redb[w][threadIdx.x];
    pb[blockIdx.x * K + threadIdx.x] = acc;
  }
}

int64_t hg_rows_per_chunk(int64_t n) {
  const int64_t want = (n + 2 * 148 - 1) / (2 * 148);
  return std::max<int64_t>(64, (want + 7) / 8 * 8);
}
int64_t hg_chunks(int64_t n) { return (n + hg_rows_per_chunk(n) - 1) / hg_rows_per_chunk(n); }

size_t rnd256(size_t b) { return (b + 255) / 256 * 256; }

int check_hg(int64_t n, int64_t d, int32_t k, int32_t mode, std::initializer_list<const void*> p,
             const char* name) {
  CIGN_REQUIRE(n >= 0 && d >= 1 && k >= 1 && k <= kMaxK, CIGN_ERR_INVALID_ARGUMENT,
               "%s: need n >= 0, d >= 1, 1 <= k <= %d", name, kMaxK);
  CIGN_REQUIRE(mode == 0 || mode == 1, CIGN_ERR_INVALID_ARGUMENT, "%s: mode must be 0 or 1",
               name);
  CIGN_REQUIRE(d % 4 == 0, CIGN_ERR_UNSUPPORTED, "%s: d must be a multiple of 4", name);
  if (n == 0) return CIGN_OK;
  for (const void* q : p) {
    CIGN_REQUIRE(q != nullptr, CIGN_ERR_NULL_POINTER, "%s: NULL argument", name);
    CIGN_REQUIRE(aligned16(q), CIGN_ERR_ALIGNMENT, "%s: tensors must be 16-byte aligned", name);
  }
  return CIGN_OK;
}

#define CIGN_HG_K_DISPATCH(k, CALL)                                 \
  switch (k) {                                                      \
    case 1: { constexpr int K_ = 1; CALL; break; }                  \
    case 2: { constexpr int K_ = 2; CALL; break; }                  \
    case 3: { constexpr int K_ = 3; CALL; break; }                  \
    case 4: { constexpr int K_ = 4; CALL; break; }                  \
    case 5: { constexpr int K_ = 5; CALL; break; }                  \
    case 6: { constexpr int K_ = 6; CALL; break; }                  \
    case 7: { constexpr int K_ = 7; CALL; break; }                  \
    default: { constexpr int K_ = 8; CALL; break; }                 \
  }

}  // namespace
}  // namespace cign

using namespace cign;

extern "C" {

int cign_hop_gate_fwd(int64_t n, int64_t d, int32_t k, int32_t mode, const float* h,
                      const float* c, const float* w, const float* b, float* alpha,
                      cign_stream_t stream) {
  int rc = check_hg(n, d, k, mode, {h, c, w}, "hop_gate_fwd");
  if (rc) return rc;
  if (n == 0) return CIGN_OK;
  CIGN_REQUIRE(b != nullptr && alpha != nullptr, CIGN_ERR_NULL_POINTER, "hop_gate_fwd: NULL");
  const int64_t blocks = (n + kThreads / 32 - 1) / (kThreads / 32);
  CIGN_REQUIRE(blocks < (1ll << 31), CIGN_ERR_UNSUPPORTED, "hop_gate_fwd: too many rows");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CIGN_HG_K_DISPATCH(k, (hop_gate_fwd_kernel<K_><<<static_cast<unsigned>(blocks), kThreads, 0, s>>>(
                            n, d, mode, h, c, w, b, alpha)));
  CIGN_CHECK_LAUNCH("hop_gate_fwd_kernel");
  return CIGN_OK;
}

size_t cign_hop_gate_bwd_workspace_bytes(int64_t n, int64_t d, int32_t k) {
  if (n <= 0 || d <= 0 || k <= 0) return 0;
  const int64_t ch = hg_chunks(n);
  return rnd256(static_cast<size_t>(ch) * k * 2 * d * sizeof(float)) +
         rnd256(static_cast<size_t>(ch) * k * sizeof(float));
}

int cign_hop_gate_bwd(int64_t n, int64_t d, int32_t k, int32_t mode, const float* h,
                      const float* c, const float* w, const float* alpha, const float* grad_alpha,
                      float* grad_h, float* grad_c, float* grad_w, float* grad_b,
                      int32_t accumulate, const float* add_h, const float* add_c, int64_t add_ld,
                      void* ws, size_t ws_bytes, cign_stream_t stream) {
  int rc = check_hg(n, d, k, mode, {h, c, w, grad_h, grad_c, ws}, "hop_gate_bwd");
  if (rc) return rc;
  CIGN_REQUIRE((add_h == nullptr && add_c == nullptr) ||
                   (add_ld >= d && add_ld % 4 == 0 && (add_h == nullptr || aligned16(add_h)) &&
                    (add_c == nullptr || aligned16(add_c))),
               CIGN_ERR_ALIGNMENT, "hop_gate_bwd: addends need 16-byte rows (add_ld % 4 == 0)");
  CIGN_REQUIRE(grad_w != nullptr && grad_b != nullptr, CIGN_ERR_NULL_POINTER,
               "hop_gate_bwd: NULL parameter gradient");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n == 0) {
    CIGN_CHECK_CUDA(cudaMemsetAsync(grad_w, 0, static_cast<size_t>(k) * 2 * d * sizeof(float), s),
                    "hop_gate_bwd: memset");
    CIGN_CHECK_CUDA(cudaMemsetAsync(grad_b, 0, static_cast<size_t>(k) * sizeof(float), s),
                    "hop_gate_bwd: memset");
    return CIGN_OK;
  }
  CIGN_REQUIRE(alpha != nullptr && grad_alpha != nullptr, CIGN_ERR_NULL_POINTER,
               "hop_gate_bwd: NULL argument");
  const size_t need = cign_hop_gate_bwd_workspace_bytes(n, d, k);
  CIGN_REQUIRE(ws_bytes >= need, CIGN_ERR_INVALID_ARGUMENT,
               "hop_gate_bwd: workspace too small (%zu < %zu bytes)", ws_bytes, need);
  const int64_t rpc = hg_rows_per_chunk(n), ch = hg_chunks(n);
  const int64_t tiles = (d + kTileCols - 1) / kTileCols;
  CIGN_REQUIRE(ch < (1ll << 31) && tiles < 65536, CIGN_ERR_UNSUPPORTED, "hop_gate_bwd: too large");
  float* pw = static_cast<float*>(ws);
  float* pb = reinterpret_cast<float*>(static_cast<char*>(ws) +
                                       rnd256(static_cast<size_t>(ch) * k * 2 * d * sizeof(float)));
  const dim3 grid(static_cast<unsigned>(ch), static_cast<unsigned>(tiles));
  CIGN_HG_K_DISPATCH(k, (hop_gate_bwd_kernel<K_><<<grid, kThreads, 0, s>>>(
                            n, d, rpc, mode, h, c, w, alpha, grad_alpha, grad_h, grad_c,
                            accumulate, add_h, add_c, add_ld, pw, pb)));
  CIGN_CHECK_LAUNCH("hop_gate_bwd_kernel");
  rc = colsum_rows(pw, grad_w, nullptr, nullptr, ch, static_cast<int64_t>(k) * 2 * d,
                   static_cast<int64_t>(k) * 2 * d, s);
  if (rc) return rc;
  return colsum_rows(pb, grad_b, nullptr, nullptr, ch, k, k, s);
}

}  // extern "C"
