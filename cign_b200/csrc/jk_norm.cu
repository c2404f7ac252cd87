// LayerNorm of the model's jumping-knowledge output, read straight from the
// per-block states: y = LN([s_0 | s_1 | ... | s_{S-1}]) with weight w and
// bias b (biased variance, y = (x - mean) * rsqrt(var + eps) * w + b), as
// GraphCliffordNet.output_norm(torch.cat(states, dim=-1))
// (generic_engine/model_cign.py:1195-1201) computes it, without the cat.
//
// Forward: one warp per row holds the row (D = S * W <= 2048 floats) in
// registers as float4 chunks; chunk c of the row is float4 (c mod W/4) of
// segment c div (W/4).  Mean and variance are two in-register passes.
// Backward: one warp per row forms grad_x = rstd * (g*w - mean(g*w) -
// xhat * mean(g*w*xhat)) in two passes and writes it back per segment; the parameter
// gradients sum g*xhat and g over rows in fixed-size row chunks (one thread
// per float4 column), then over chunks with colsum_rows: fixed order, no
// atomics.
#include <algorithm>

#include "common.cuh"

namespace cign {
namespace {

constexpr int kJkThreads = 256;
constexpr int kJkWarps = kJkThreads / 32;
constexpr int kJkMaxSeg = 8;
constexpr int kJkRowsPerChunk = 64;

struct SegPtrs { const float* p[kJkMaxSeg]; };
struct SegOut { float* p[kJkMaxSeg]; };

// Segment `seg`'s base pointer by a chain of selects: indexing the parameter
// array with a run-time index would copy it to local memory.
template <typename P>
__device__ __forceinline__ auto seg_base(const P& s, int seg) -> decltype(s.p[0]) {
  auto q = s.p[0];
#pragma unroll
  for (int i = 1; i < kJkMaxSeg; ++i)
    if (seg == i) q = s.p[i];
  return q;
}

// Walks a lane's float4 columns c = lane, lane + 32, ... of the row as
// (segment, column within the segment) without dividing by the segment width.
struct SegCursor {
  int seg;
  int cs;
  __device__ __forceinline__ SegCursor(int lane, int wq) : seg(0), cs(lane) {
    while (cs >= wq) { cs -= wq; ++seg; }
  }
  __device__ __forceinline__ void next(int wq) {
    cs += 32;
    while (cs >= wq) { cs -= wq; ++seg; }
  }
};

template <int NCH>
__global__ void __launch_bounds__(kJkThreads)
jk_ln_fwd_kernel(int64_t n, int64_t W, int64_t D, SegPtrs segs, const float* __restrict__ w,
                 const float* __restrict__ b, float eps, float* __restrict__ y,
                 float* __restrict__ mean, float* __restrict__ rstd) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kJkWarps + (threadIdx.x >> 5);
  if (row >= n) return;
  const int wq = static_cast<int>(W / 4);  // float4 chunks per segment
  const int64_t dq = D / 4;
  float4 x[NCH];
  float s = 0.0f;
  SegCursor cur(lane, wq);
#pragma unroll
  for (int k = 0; k < NCH; ++k) {
    const int64_t c = lane + 32 * k;
    x[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (c < dq) {
      x[k] = __ldg(reinterpret_cast<const float4*>(seg_base(segs, cur.seg) + row * W) + cur.cs);
      s += (x[k].x + x[k].y) + (x[k].z + x[k].w);
    }
    cur.next(wq);
  }
  const float mu = warp_sum(s) / static_cast<float>(D);
  float v = 0.0f;
#pragma unroll
  for (int k = 0; k < NCH; ++k) {
    const int64_t c = lane + 32 * k;
    if (c < dq) {
      const float a0 = x[k].x - mu, a1 = x[k].y - mu, a2 = x[k].z - mu, a3 = x[k].w - mu;
      v += (a0 * a0 + a1 * a1) + (a2 * a2 + a3 * a3);
    }
  }
  const float rs = rsqrtf(warp_sum(v) / static_cast<float>(D) + eps);
  if (lane == 0) {
    mean[row] = mu;
    rstd[row] = rs;
  }
#pragma unroll
  for (int k = 0; k < NCH; ++k) {
    const int64_t c = lane + 32 * k;
    if (c < dq) {
      const float4 wv = __ldg(reinterpret_cast<const float4*>(w) + c);
      const float4 bv = __ldg(reinterpret_cast<const float4*>(b) + c);
      float4 o;
      o.x = (x[k].x - mu) * rs * wv.x + bv.x;
      o.y = (x[k].y - mu) * rs * wv.y + bv.y;
      o.z = (x[k].z - mu) * rs * wv.z + bv.z;
      o.w = (x[k].w - mu) * rs * wv.w + bv.w;
      reinterpret_cast<float4*>(y + row * D)[c] = o;
    }
  }
}

// Two passes over the row: the first forms the row sums of g*w and g*w*xhat,
// the second reloads x, g, w (L1 hits) and writes grad_x, so a lane holds no
// row arrays and the kernel keeps enough warps resident to cover the loads.
template <int NCH>
__global__ void __launch_bounds__(kJkThreads)
jk_ln_bwd_kernel(int64_t n, int64_t W, int64_t D, const float* __restrict__ gy, SegPtrs segs,
                 const float* __restrict__ w, const float* __restrict__ mean,
                 const float* __restrict__ rstd, SegOut gsegs) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kJkWarps + (threadIdx.x >> 5);
  if (row >= n) return;
  const int wq = static_cast<int>(W / 4);
  const int64_t dq = D / 4;
  const float mu = mean[row], rs = rstd[row];
  float s1 = 0.0f, s2 = 0.0f;
  SegCursor cur(lane, wq);
#pragma unroll 4
  for (int k = 0; k < NCH; ++k, cur.next(wq)) {
    const int64_t c = lane + 32 * k;
    if (c < dq) {
      const float4 xv =
          __ldg(reinterpret_cast<const float4*>(seg_base(segs, cur.seg) + row * W) + cur.cs);
      const float4 gv = __ldg(reinterpret_cast<const float4*>(gy + row * D) + c);
      const float4 wv = __ldg(reinterpret_cast<const float4*>(w) + c);
      const float d0 = gv.x * wv.x, d1 = gv.y * wv.y, d2 = gv.z * wv.z, d3 = gv.w * wv.w;
      s1 += (d0 + d1) + (d2 + d3);
      s2 += (d0 * ((xv.x - mu) * rs) + d1 * ((xv.y - mu) * rs)) +
            (d2 * ((xv.z - mu) * rs) + d3 * ((xv.w - mu) * rs));
    }
  }
  const float Df = static_cast<float>(D);
  s1 = warp_sum(s1);
  s2 = warp_sum(s2);
  const float f = rs / Df;
  SegCursor cur2(lane, wq);
#pragma unroll 4
  for (int k = 0; k < NCH; ++k, cur2.next(wq)) {
    const int64_t c = lane + 32 * k;
    if (c < dq) {
      const float4 xv =
          __ldg(reinterpret_cast<const float4*>(seg_base(segs, cur2.seg) + row * W) + cur2.cs);
      const float4 gv = __ldg(reinterpret_cast<const float4*>(gy + row * D) + c);
      const float4 wv = __ldg(reinterpret_cast<const float4*>(w) + c);
      float4 o;
      o.x = f * (Df * (gv.x * wv.x) - s1 - ((xv.x - mu) * rs) * s2);
      o.y = f * (Df * (gv.y * wv.y) - s1 - ((xv.y - mu) * rs) * s2);
      o.z = f * (Df * (gv.z * wv.z) - s1 - ((xv.z - mu) * rs) * s2);
      o.w = f * (Df * (gv.w * wv.w) - s1 - ((xv.w - mu) * rs) * s2);
      reinterpret_cast<float4*>(seg_base(gsegs, cur2.seg) + row * W)[cur2.cs] = o;
    }
  }
}

// Column partials over one chunk of kJkRowsPerChunk rows: pw[chunk][d] =
// sum gy*xhat, pb[chunk][d] = sum gy, rows in order.  Eight rows' loads
// are issued together per thread (the sums still add the rows in order),
// and 128-thread blocks leave no idle threads at the 384 float4 columns of a
// 3 x 512 JK row.
constexpr int kJkParamThreads = 128;
__global__ void __launch_bounds__(kJkParamThreads)
jk_ln_param_kernel(int64_t n, int64_t W, int64_t D, const float* __restrict__ gy, SegPtrs segs,
                   const float* __restrict__ mean, const float* __restrict__ rstd,
                   float* __restrict__ pw, float* __restrict__ pb) {
  const int64_t c = static_cast<int64_t>(blockIdx.y) * kJkParamThreads + threadIdx.x;  // float4 col
  const int64_t dq = D / 4;
  if (c >= dq) return;
  const int64_t wq = W / 4;
  const int seg = static_cast<int>(c / wq);
  const float4* xs = reinterpret_cast<const float4*>(seg_base(segs, seg)) + (c - seg * wq);
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kJkRowsPerChunk;
  const int64_t r1 = r0 + kJkRowsPerChunk < n ? r0 + kJkRowsPerChunk : n;
  float4 aw = make_float4(0.f, 0.f, 0.f, 0.f), ab = aw;
  constexpr int kG = 8;  // rows whose loads are issued together
  for (int64_t rb = r0; rb < r1; rb += kG) {
    float4 xv[kG], gv[kG];
    float mu[kG], rs[kG];
#pragma unroll
    for (int u = 0; u < kG; ++u) {
      const int64_t r = rb + u < r1 ? rb + u : r1 - 1;  // clamped: loaded, not added
      mu[u] = __ldg(mean + r);
      rs[u] = __ldg(rstd + r);
      xv[u] = __ldg(xs + r * wq);
      gv[u] = __ldg(reinterpret_cast<const float4*>(gy + r * D) + c);
    }
#pragma unroll
    for (int u = 0; u < kG; ++u) {
      if (rb + u >= r1) break;
      aw.x += gv[u].x * ((xv[u].x - mu[u]) * rs[u]);
      aw.y += gv[u].y * ((xv[u].y - mu[u]) * rs[u]);
      aw.z += gv[u].z * ((xv[u].z - mu[u]) * rs[u]);
      aw.w += gv[u].w * ((xv[u].w - mu[u]) * rs[u]);
      ab.x += gv[u].x;
      ab.y += gv[u].y;
      ab.z += gv[u].z;
      ab.w += gv[u].w;
    }
  }
  reinterpret_cast<float4*>(pw + static_cast<int64_t>(blockIdx.x) * D)[c] = aw;
  reinterpret_cast<float4*>(pb + static_cast<int64_t>(blockIdx.x) * D)[c] = ab;
}

int64_t jk_chunks(int64_t n) { return (n + kJkRowsPerChunk - 1) / kJkRowsPerChunk; }

int jk_check(int64_t n, int32_t n_seg, int64_t W, const char* name) {
  CIGN_REQUIRE(n >= 0 && W > 0, CIGN_ERR_INVALID_ARGUMENT, "%s: bad sizes", name);
  CIGN_REQUIRE(n_seg >= 1 && n_seg <= kJkMaxSeg, CIGN_ERR_UNSUPPORTED,
               "%s: 1..%d segments supported", name, kJkMaxSeg);
  CIGN_REQUIRE(W % 4 == 0 && n_seg * W <= 2048, CIGN_ERR_UNSUPPORTED,
               "%s: segment width must be a multiple of 4 and the row at most 2048 floats",
               name);
  CIGN_REQUIRE(n < (1ll << 31) * kJkWarps, CIGN_ERR_UNSUPPORTED, "%s: too many rows", name);
  return CIGN_OK;
}

#define CIGN_JK_DISPATCH(D, CALL)                 \
  do {                                            \
    const int64_t nch_ = ((D) / 4 + 31) / 32;     \
    if (nch_ <= 4) { constexpr int NCH = 4; CALL; } \
    else if (nch_ <= 8) { constexpr int NCH = 8; CALL; } \
    else if (nch_ <= 12) { constexpr int NCH = 12; CALL; } \
    else { constexpr int NCH = 16; CALL; }        \
  } while (0)

}  // namespace
}  // namespace cign

using namespace cign;

extern "C" {

size_t cign_jk_ln_workspace_bytes(int64_t n, int64_t d) {
  if (n <= 0 || d <= 0) return 0;
  return 2 * static_cast<size_t>(jk_chunks(n)) * d * sizeof(float);
}

int cign_jk_ln_fwd(int64_t n, int32_t n_seg, int64_t seg_width, const float* const* segs,
                   const float* w, const float* b, float eps, float* y, float* mean, float* rstd,
                   cign_stream_t stream) {
  int rc = jk_check(n, n_seg, seg_width, "jk_ln_fwd");
  if (rc) return rc;
  if (n == 0) return CIGN_OK;
  CIGN_REQUIRE(segs && w && b && y && mean && rstd, CIGN_ERR_NULL_POINTER,
               "jk_ln_fwd: NULL argument");
  SegPtrs P{};
  for (int i = 0; i < n_seg; ++i) {
    CIGN_REQUIRE(segs[i] != nullptr && aligned16(segs[i]), CIGN_ERR_ALIGNMENT,
                 "jk_ln_fwd: segment %d must be a 16-byte aligned device pointer", i);
    P.p[i] = segs[i];
  }
  CIGN_REQUIRE(aligned16(w) && aligned16(b) && aligned16(y), CIGN_ERR_ALIGNMENT,
               "jk_ln_fwd: w, b, y must be 16-byte aligned");
  const int64_t D = n_seg * seg_width;
  const unsigned grid = static_cast<unsigned>((n + kJkWarps - 1) / kJkWarps);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CIGN_JK_DISPATCH(D, (jk_ln_fwd_kernel<NCH><<<grid, kJkThreads, 0, s>>>(
                          n, seg_width, D, P, w, b, eps, y, mean, rstd)));
  CIGN_CHECK_LAUNCH("jk_ln_fwd_kernel");
  return CIGN_OK;
}

int cign_jk_ln_bwd(int64_t n, int32_t n_seg, int64_t seg_width, const float* grad_y,
                   const float* const* segs, const float* w, const float* mean,
                   const float* rstd, float* const* grad_segs, float* grad_w, float* grad_b,
                   void* ws, size_t ws_bytes, cign_stream_t stream) {
  int rc = jk_check(n, n_seg, seg_width, "jk_ln_bwd");
  if (rc) return rc;
  const int64_t D = n_seg * seg_width;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CIGN_REQUIRE(grad_w && grad_b, CIGN_ERR_NULL_POINTER, "jk_ln_bwd: NULL argument");
  if (n == 0) {
    CIGN_CHECK_CUDA(cudaMemsetAsync(grad_w, 0, D * sizeof(float), s), "jk_ln_bwd: memset");
    CIGN_CHECK_CUDA(cudaMemsetAsync(grad_b, 0, D * sizeof(float), s), "jk_ln_bwd: memset");
    return CIGN_OK;
  }
  CIGN_REQUIRE(grad_y && segs && w && mean && rstd && grad_segs && ws, CIGN_ERR_NULL_POINTER,
               "jk_ln_bwd: NULL argument");
  const size_t need = cign_jk_ln_workspace_bytes(n, D);
  CIGN_REQUIRE(ws_bytes >= need, CIGN_ERR_INVALID_ARGUMENT,
               "jk_ln_bwd: workspace too small (%zu < %zu bytes)", ws_bytes, need);
  SegPtrs P{};
  SegOut G{};
  for (int i = 0; i < n_seg; ++i) {
    CIGN_REQUIRE(segs[i] != nullptr && grad_segs[i] != nullptr && aligned16(segs[i]) &&
                     aligned16(grad_segs[i]),
                 CIGN_ERR_ALIGNMENT, "jk_ln_bwd: segment %d must be 16-byte aligned", i);
    P.p[i] = segs[i];
    G.p[i] = grad_segs[i];
  }
  CIGN_REQUIRE(aligned16(grad_y) && aligned16(w) && aligned16(ws), CIGN_ERR_ALIGNMENT,
               "jk_ln_bwd: grad_y, w, ws must be 16-byte aligned");
  const unsigned grid = static_cast<unsigned>((n + kJkWarps - 1) / kJkWarps);
  CIGN_JK_DISPATCH(D, (jk_ln_bwd_kernel<NCH><<<grid, kJkThreads, 0, s>>>(
                          n, seg_width, D, grad_y, P, w, mean, rstd, G)));
  CIGN_CHECK_LAUNCH("jk_ln_bwd_kernel");
  const int64_t chunks = jk_chunks(n);
  float* pw = static_cast<float*>(ws);
  float* pb = pw + chunks * D;
  const dim3 pgrid(static_cast<unsigned>(chunks),
                   static_cast<unsigned>((D / 4 + kJkParamThreads - 1) / kJkParamThreads));
  jk_ln_param_kernel<<<pgrid, kJkParamThreads, 0, s>>>(n, seg_width, D, grad_y, P, mean, rstd,
                                                        pw, pb);
  CIGN_CHECK_LAUNCH("jk_ln_param_kernel");
  return colsum_rows(pw, grad_w, pb, grad_b, chunks, D, D, s);
}

}  // extern "C"
