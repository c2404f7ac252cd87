// Collapsed multi-head GAT (concat=False) for sm_100a: edge logits,
// LeakyReLU, segment softmax, attention dropout, weighted aggregation, head
// mean, bias and SiLU in one CSR pass; backward in two graph passes.
//
// Reference: collapsed_gat_ext/collapsed_gat_cuda.cu (forward :52-174, grad
// kernels :176-430, host :434-545) behind collapsed_gat.py:57-225.
//
// Layout: destination-major CSR (rowptr, col) and its CSC (colptr, row) with
// perm[csc position] = CSR edge id, in_feat [N,H,C], attn_* [N,H].
//
// Work split: rows (and, in the backward, CSC columns) with at most kSegLen
// edges are processed whole by one group of LPR lanes; longer "hub" rows are
// cut at plan time into kSegLen-edge segments, one group each, whose partial
// results are combined by a per-hub kernel in segment order (fixed sum
// order: deterministic).
//
// Forward, per destination row i:
//   1. per head h: max and exp-sum of e_ij = leaky(attn_row[i,h] +
//      attn_col[j,h]) (group reductions; hub rows: one CTA per row first);
//   2. per 32-edge chunk and head: the lane owning edge e computes its weight
//      w = keep(e*H+h) * exp(e_ij - max) / sum / (1-p) once, the group
//      broadcasts (col, w) and accumulates w * in_feat[j,h,:] into the row's
//      C-wide register tile (heads summed into one tile: "collapsed");
//   3. pre = acc / H + bias, out = SiLU(pre).
// The dropout mask is a pure function of (seed, e*H+h) and is recomputed in
// backward instead of being stored.
//
// Backward:
//   K1 (CSR rows): g_pre = grad_y * SiLU'(pre) (workspace); per edge and head
//      dot(g_pre[i,:]/H, in_feat[j,h,:]); softmax backward through the
//      kept/scaled weights and LeakyReLU -> grad_logit[e,h] (workspace) and
//      grad_attn_row[i,h] (row sums; hub rows finish in a per-row CTA).
//   K2 (CSC columns): grad_feat[j,h,:] = sum_{i->j} w_ijh g_pre[i,:]/H and
//      grad_attn_col[j,h] = sum_{i->j} grad_logit[e,h] -- gathers, so no
//      atomics anywhere.
//   grad_bias = column sums of g_pre (two-stage, fixed order).
#include <cuda_bf16.h>

#include <algorithm>
#include <initializer_list>
#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"

struct cign_gat_plan {
  int64_t n;       // destination rows (CSR rows)
  int64_t n_cols;  // source columns (CSC columns); == n for a square graph
  int64_t nnz;
  const int32_t* rowptr;
  const int32_t* col;
  const int32_t* colptr;
  const int32_t* row;
  const int32_t* perm;
  cign::SegList rows;  // hub destination rows (CSR)
  cign::SegList cols;  // hub source columns (CSC)
  // the same with kAggSegLen-edge work items, for the aggregate-first
  // aggregation kernels (gat_agg_kernel walks an item in 32-edge chunks)
  cign::SegList agg_rows;
  cign::SegList agg_cols;
  int device;
};

namespace cign {
namespace {

constexpr int kThreads = 256;
constexpr int kSegLen = 32;
constexpr int kMaxHeads = 64;
constexpr float kNegInit = -1.0e38f;  // reference initial running max

template <int VEC, int VPL, int LPR>
struct GatCfg {
  static constexpr int kGroups = kThreads / LPR;
  static constexpr int kTile = LPR * VPL * VEC;
  static constexpr int kUnroll = VPL >= 8 ? 2 : 4;
};

template <int LPR>
__device__ __forceinline__ float group_sum(float v, unsigned gmask) {
#pragma unroll
  for (int o = LPR / 2; o > 0; o >>= 1) v += __shfl_xor_sync(gmask, v, o, LPR);
  return v;
}
template <int LPR>
__device__ __forceinline__ float group_max(float v, unsigned gmask) {
#pragma unroll
  for (int o = LPR / 2; o > 0; o >>= 1)
    v = fmaxf(v, __shfl_xor_sync(gmask, v, o, LPR));
  return v;
}

template <int LPR>
__device__ __forceinline__ unsigned group_mask() {
  return LPR == 32 ? kFullMask
                   : (((1u << LPR) - 1u) << ((threadIdx.x & 31) / LPR * LPR));
}

// Block-wide reductions over kThreads threads (all threads must call).
template <int NT = kThreads>
__device__ __forceinline__ float block_sum(float v, float* scratch) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) scratch[w] = v;
  __syncthreads();
  float r = 0.0f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) r += scratch[i];
  return r;
}
template <int NT = kThreads>
__device__ __forceinline__ float block_max(float v, float* scratch) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) scratch[w] = v;
  __syncthreads();
  float r = scratch[0];
#pragma unroll
  for (int i = 1; i < NT / 32; ++i) r = fmaxf(r, scratch[i]);
  return r;
}

// Attention weight of CSR edge e (head h) as the reference forms it:
// w = exp(leaky(ad + ac) - m) / s, divided by (1 - p) when p > 0; zero when
// the edge is dropped or the row sum is not positive.
__device__ __forceinline__ float edge_weight(float ad, float ac, float m, float s, float slope,
                                             float p, uint64_t seed, uint64_t idx) {
  const bool keep = (p <= 0.0f) || gat_keep(seed, idx, p);
  if (!keep || !(s > 0.0f)) return 0.0f;
  float w = expf(leaky_f(ad + ac, slope) - m) / s;
  if (p > 0.0f) w /= (1.0f - p);
  return w;
}

// acc[q] += sum over edges [e0, e1) and all heads of
// w(e,h) * in_feat[col[e], h, f0 + (lig + q*LPR)*VEC ...]; smax/ssum point at
// the row's per-head max and exp-sum.
template <int VEC, int VPL, int LPR>
__device__ __forceinline__ void gat_gather(
    int64_t row, int e0, int e1, int H, int64_t C, int64_t f0, const int* __restrict__ col,
    const float* __restrict__ attn_row, const float* __restrict__ attn_col,
    const float* __restrict__ x, const float* smax, const float* ssum, float slope, float p,
    uint64_t seed, int lig, unsigned gmask, typename VecT<VEC>::type (&acc)[VPL]) {
  using V = typename VecT<VEC>::type;
  using Cfg = GatCfg<VEC, VPL, LPR>;
  const int64_t HC = static_cast<int64_t>(H) * C;
  for (int base = e0; base < e1; base += LPR) {
    const int my = base + lig;
    const bool valid = my < e1;
    const int c = valid ? __ldg(col + my) : 0;
    const int cnt = min(LPR, e1 - base);
    for (int h = 0; h < H; ++h) {
      float w = 0.0f;
      if (valid)
        w = edge_weight(__ldg(attn_row + row * H + h),
                        __ldg(attn_col + static_cast<int64_t>(c) * H + h), smax[h], ssum[h],
                        slope, p, seed, static_cast<uint64_t>(my) * H + h);
      const float* xh = x + static_cast<int64_t>(h) * C + f0;
      int t = 0;
      for (; t + Cfg::kUnroll <= cnt; t += Cfg::kUnroll) {
        int cc[Cfg::kUnroll];
        float ww[Cfg::kUnroll];
#pragma unroll
        for (int u = 0; u < Cfg::kUnroll; ++u) {
          cc[u] = __shfl_sync(gmask, c, t + u, LPR);
          ww[u] = __shfl_sync(gmask, w, t + u, LPR);
        }
        V xv[Cfg::kUnroll][VPL];
#pragma unroll
        for (int u = 0; u < Cfg::kUnroll; ++u) {
          const float* xr = xh + static_cast<int64_t>(cc[u]) * HC;
#pragma unroll
          for (int q = 0; q < VPL; ++q) {
            const int64_t fi = static_cast<int64_t>(lig + q * LPR) * VEC;
            if (f0 + fi < C) xv[u][q] = ldg_vec<VEC>(xr + fi);
            else vzero(xv[u][q]);
          }
        }
#pragma unroll
        for (int u = 0; u < Cfg::kUnroll; ++u)
#pragma unroll
          for (int q = 0; q < VPL; ++q) vfma(acc[q], ww[u], xv[u][q]);
      }
      for (; t < cnt; ++t) {
        const int c0 = __shfl_sync(gmask, c, t, LPR);
        const float w0 = __shfl_sync(gmask, w, t, LPR);
        const float* xr = xh + static_cast<int64_t>(c0) * HC;
#pragma unroll
        for (int q = 0; q < VPL; ++q) {
          const int64_t fi = static_cast<int64_t>(lig + q * LPR) * VEC;
          if (f0 + fi < C) vfma(acc[q], w0, ldg_vec<VEC>(xr + fi));
        }
      }
    }
  }
}

// ------------------------------------------------------------ forward
// Hub rows: CTA (hub, head) of kHubThreads threads computes that head's
// max / exp-sum of the row.  The largest hub of a power-law graph (thousands
// of edges) sets these kernels' time: measured on the cfg2 graph, two-warp
// CTAs took 2.8x longer than eight-warp ones despite fitting every hub in
// one wave.
constexpr int kHubThreads = kThreads;
constexpr int kHubBatch = 4;  // edges per thread whose loads are in flight together
__global__ void __launch_bounds__(kHubThreads)
gat_hub_stats_kernel(int H, const int* __restrict__ rowptr, const int* __restrict__ col,
                     const int* __restrict__ hub_row, const float* __restrict__ attn_row,
                     const float* __restrict__ attn_col, float slope,
                     float* __restrict__ emax, float* __restrict__ esum) {
  __shared__ float scratch[32];
  const int64_t row = hub_row[blockIdx.x];
  const int h = blockIdx.y;
  const int e0 = rowptr[row], e1 = rowptr[row + 1];
  const float ad = attn_row[row * H + h];
  // edges in groups of kHubBatch per thread with their loads issued
  // together; the per-thread max and sum still run over the edges in order
  float m = kNegInit;
  for (int eb = e0 + threadIdx.x; eb < e1; eb += kHubBatch * kHubThreads) {
    float ac[kHubBatch];
#pragma unroll
    for (int u = 0; u < kHubBatch; ++u) {
      const int e = eb + u * kHubThreads;
      ac[u] = e < e1 ? attn_col[static_cast<int64_t>(col[e]) * H + h] : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < kHubBatch; ++u)
      if (eb + u * kHubThreads < e1) m = fmaxf(m, leaky_f(ad + ac[u], slope));
  }
  m = block_max<kHubThreads>(m, scratch);
  float s = 0.0f;
  for (int eb = e0 + threadIdx.x; eb < e1; eb += kHubBatch * kHubThreads) {
    float ac[kHubBatch];
#pragma unroll
    for (int u = 0; u < kHubBatch; ++u) {
      const int e = eb + u * kHubThreads;
      ac[u] = e < e1 ? attn_col[static_cast<int64_t>(col[e]) * H + h] : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < kHubBatch; ++u)
      if (eb + u * kHubThreads < e1) s += expf(leaky_f(ad + ac[u], slope) - m);
  }
  s = block_sum<kHubThreads>(s, scratch);
  if (threadIdx.x == 0) {
    emax[row * H + h] = m;
    esum[row * H + h] = s;
  }
}

// Blocks [0, seg_blocks): hub-row segments -> partial [n_seg, C];
// remaining blocks: whole rows of at most kSegLen edges.
template <int VEC, int VPL, int LPR>
__global__ void __launch_bounds__(kThreads)
gat_fwd_kernel(int n, int H, int64_t C, const int* __restrict__ rowptr,
               const int* __restrict__ col, const int* __restrict__ seg_row,
               const int* __restrict__ seg_begin, const int* __restrict__ seg_end, int n_seg,
               int seg_blocks, const float* __restrict__ attn_row,
               const float* __restrict__ attn_col, const float* __restrict__ x,
               const float* __restrict__ bias, float slope, float p, Seed seed_in,
               float* __restrict__ out, float* __restrict__ pre, float* __restrict__ emax,
               float* __restrict__ esum, float* __restrict__ partial) {
  const uint64_t seed = seed_in;
  using V = typename VecT<VEC>::type;
  using Cfg = GatCfg<VEC, VPL, LPR>;
  extern __shared__ float smem[];  // [kGroups][2H] row statistics
  const int lig = threadIdx.x % LPR;
  const int group = threadIdx.x / LPR;
  const unsigned gmask = group_mask<LPR>();

  if (static_cast<int>(blockIdx.x) < seg_blocks) {
    const int64_t sidx = static_cast<int64_t>(blockIdx.x) * Cfg::kGroups + group;
    if (sidx >= n_seg) return;
    const int64_t row = seg_row[sidx];
    const int e0 = seg_begin[sidx], e1 = seg_end[sidx];
    for (int64_t f0 = 0; f0 < C; f0 += Cfg::kTile) {
      V acc[VPL];
#pragma unroll
      for (int q = 0; q < VPL; ++q) vzero(acc[q]);
      gat_gather<VEC, VPL, LPR>(row, e0, e1, H, C, f0, col, attn_row, attn_col, x,
                                emax + row * H, esum + row * H, slope, p, seed, lig, gmask, acc);
#pragma unroll
      for (int q = 0; q < VPL; ++q) {
        const int64_t fi = static_cast<int64_t>(lig + q * LPR) * VEC;
        if (f0 + fi < C) st_vec(partial + sidx * C + f0 + fi, acc[q]);
      }
    }
    return;
  }

  const int64_t row64 = static_cast<int64_t>(blockIdx.x - seg_blocks) * Cfg::kGroups + group;
  if (row64 >= n) return;
  const int e0 = rowptr[row64], e1 = rowptr[row64 + 1];
  if (e1 - e0 > kSegLen) return;  // hub row: stats, segments and combine kernels
  float* stats = smem + group * 2 * H;
  for (int h = 0; h < H; ++h) {
    const float ad = attn_row[row64 * H + h];
    float m = kNegInit;
    for (int e = e0 + lig; e < e1; e += LPR)
      m = fmaxf(m, leaky_f(ad + attn_col[static_cast<int64_t>(col[e]) * H + h], slope));
    m = group_max<LPR>(m, gmask);
    float s = 0.0f;
    for (int e = e0 + lig; e < e1; e += LPR)
      s += expf(leaky_f(ad + attn_col[static_cast<int64_t>(col[e]) * H + h], slope) - m);
    s = group_sum<LPR>(s, gmask);
    if (lig == 0) {
      stats[h] = m;
      stats[H + h] = s;
      emax[row64 * H + h] = m;
      esum[row64 * H + h] = s;
    }
  }
  __syncwarp(gmask);
  const float hf = static_cast<float>(H);
  for (int64_t f0 = 0; f0 < C; f0 += Cfg::kTile) {
    V acc[VPL];
#pragma unroll
    for (int q = 0; q < VPL; ++q) vzero(acc[q]);
    gat_gather<VEC, VPL, LPR>(row64, e0, e1, H, C, f0, col, attn_row, attn_col, x, stats,
                              stats + H, slope, p, seed, lig, gmask, acc);
#pragma unroll
    for (int q = 0; q < VPL; ++q) {
      const int64_t fi = static_cast<int64_t>(lig + q * LPR) * VEC;
      if (f0 + fi < C) {
        V pv, ov;
        const V bv = ldg_vec<VEC>(bias + f0 + fi);
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          const float pj = vel(acc[q], j) / hf + vel(bv, j);
          vel(pv, j) = pj;
          vel(ov, j) = silu_f(pj);
        }
        st_vec(pre + row64 * C + f0 + fi, pv);
        st_vec(out + row64 * C + f0 + fi, ov);
      }
    }
  }
}

// Hub-row combine: acc = sum of the row's segment partials (segment order),
// pre = acc / H + bias, out = SiLU(pre).  Block (hub, chunk) covers
// kCombineThreads * VEC channels.
constexpr int kCombineThreads = 64;

template <int VEC>
__global__ void __launch_bounds__(kCombineThreads)
gat_fwd_combine_kernel(int H, int64_t C, const int* __restrict__ hub_row,
                       const int* __restrict__ hub_first, const float* __restrict__ partial,
                       const float* __restrict__ bias, float* __restrict__ pre,
                       float* __restrict__ out) {
  using V = typename VecT<VEC>::type;
  const int64_t c = (static_cast<int64_t>(blockIdx.y) * kCombineThreads + threadIdx.x) * VEC;
  if (c >= C) return;
  const int64_t row = hub_row[blockIdx.x];
  const V a = ordered_sum<VEC>(partial + c, C, hub_first[blockIdx.x], hub_first[blockIdx.x + 1]);
  const V bv = ld_vec<VEC>(bias + c);
  const float hf = static_cast<float>(H);
  V pv, ov;
#pragma unroll
  for (int j = 0; j < VEC; ++j) {
    const float pj = vel(a, j) / hf + vel(bv, j);
    vel(pv, j) = pj;
    vel(ov, j) = silu_f(pj);
  }
  st_vec(pre + row * C + c, pv);
  st_vec(out + row * C + c, ov);
}

// ------------------------------------------------------------ backward K1
// Loads grad_y/pre of one row tile, optionally writes g_pre (unscaled) and
// returns g_pre / H in registers.
template <int VEC, int VPL, int LPR>
__device__ __forceinline__ void k1_gpre(int64_t row, int64_t C, int64_t f0, int H, int lig,
                                        bool write, const float* __restrict__ grad_y,
                                        const float* __restrict__ pre, float* __restrict__ gpre,
                                        typename VecT<VEC>::type (&g)[VPL]) {
  const float inv_h = 1.0f / static_cast<float>(H);
#pragma unroll
  for (int q = 0; q < VPL; ++q) {
    const int64_t fi = static_cast<int64_t>(lig + q * LPR) * VEC;
    if (f0 + fi < C) {
      const auto gy = ld_vec<VEC>(grad_y + row * C + f0 + fi);
      const auto pr = ld_vec<VEC>(pre + row * C + f0 + fi);
      typename VecT<VEC>::type gp;
#pragma unroll
      for (int j = 0; j < VEC; ++j) vel(gp, j) = vel(gy, j) * silu_grad_f(vel(pr, j));
      if (write) st_vec(gpre + row * C + f0 + fi, gp);
#pragma unroll
      for (int j = 0; j < VEC; ++j) vel(g[q], j) = vel(gp, j) * inv_h;
    } else {
      vzero(g[q]);
    }
  }
}

// dots d(e,h) = sum_c g[c] x[col[e],h,c] over this tile for edges [e0, e1);
// the lane owning edge e stores (first tile) or adds (later tiles) glog[e,h].
template <int VEC, int VPL, int LPR>
__device__ __forceinline__ void k1_dots(int e0, int e1, int H, int64_t C, int64_t f0,
                                        bool first_tile, const int* __restrict__ col,
                                        const float* __restrict__ x,
                                        const typename VecT<VEC>::type (&g)[VPL], int lig,
                                        unsigned gmask, float* __restrict__ glog) {
  using V = typename VecT<VEC>::type;
  const int64_t HC = static_cast<int64_t>(H) * C;
  for (int base = e0; base < e1; base += LPR) {
    const int my = base + lig;
    const bool valid = my < e1;
    const int c = valid ? __ldg(col + my) : 0;
    const int cnt = min(LPR, e1 - base);
    for (int h = 0; h < H; ++h) {
      const float* xh = x + static_cast<int64_t>(h) * C + f0;
      float mine = 0.0f;
      int t = 0;
      for (; t + 2 <= cnt; t += 2) {
        const int c0 = __shfl_sync(gmask, c, t, LPR);
        const int c1 = __shfl_sync(gmask, c, t + 1, LPR);
        V x0[VPL], x1[VPL];
#pragma unroll
        for (int q = 0; q < VPL; ++q) {
          const int64_t fi = static_cast<int64_t>(lig + q * LPR) * VEC;
          if (f0 + fi < C) {
            x0[q] = ldg_vec<VEC>(xh + static_cast<int64_t>(c0) * HC + fi);
            x1[q] = ldg_vec<VEC>(xh + static_cast<int64_t>(c1) * HC + fi);
          } else {
            vzero(x0[q]);
            vzero(x1[q]);
          }
        }
        float d0 = 0.0f, d1 = 0.0f;
#pragma unroll
        for (int q = 0; q < VPL; ++q)
#pragma unroll
          for (int j = 0; j < VEC; ++j) {
            d0 = fmaf(vel(g[q], j), vel(x0[q], j), d0);
            d1 = fmaf(vel(g[q], j), vel(x1[q], j), d1);
          }
        d0 = group_sum<LPR>(d0, gmask);
        d1 = group_sum<LPR>(d1, gmask);
        if (lig == t) mine = d0;
        if (lig == t + 1) mine = d1;
      }
      for (; t < cnt; ++t) {
        const int c0 = __shfl_sync(gmask, c, t, LPR);
        float d0 = 0.0f;
#pragma unroll
        for (int q = 0; q < VPL; ++q) {
          const int64_t fi = static_cast<int64_t>(lig + q * LPR) * VEC;
          if (f0 + fi < C) {
            const V xv = ldg_vec<VEC>(xh + static_cast<int64_t>(c0) * HC + fi);
#pragma unroll
            for (int j = 0; j < VEC; ++j) d0 = fmaf(vel(g[q], j), vel(xv, j), d0);
          }
        }
        d0 = group_sum<LPR>(d0, gmask);
        if (lig == t) mine = d0;
      }
      if (valid) {
        const int64_t o = static_cast<int64_t>(my) * H + h;
        glog[o] = first_tile ? mine : glog[o] + mine;
      }
    }
  }
}

// Softmax/dropout/LeakyReLU backward of one edge (reference
// attention_backward_kernel, collapsed_gat_cuda.cu:362-430).
struct EdgeSoft {
  float soft;  // exp(leaky(raw) - m)/s  (0 when s <= 0)
  float ge;    // kept and rescaled upstream gradient of the weight
  bool neg;    // raw < 0 (LeakyReLU slope branch)
};
__device__ __forceinline__ EdgeSoft edge_soft(float ad, float ac, float m, float s, float slope,
                                              float p, uint64_t seed, uint64_t idx, float dot) {
  EdgeSoft r;
  const float raw = ad + ac;
  r.neg = raw < 0.0f;
  r.soft = s > 0.0f ? expf(leaky_f(raw, slope) - m) / s : 0.0f;
  const bool keep = (p <= 0.0f) || gat_keep(seed, idx, p);
  float ge = keep ? dot : 0.0f;
  if (p > 0.0f) ge /= (1.0f - p);
  r.ge = ge;
  return r;
}

// Blocks [0, seg_blocks): hub-row segments compute their edges' dots;
// remaining blocks: whole rows (g_pre, dots, softmax backward).
template <int VEC, int VPL, int LPR>
__global__ void __launch_bounds__(kThreads)
gat_bwd_rows_kernel(int n, int H, int64_t C, const int* __restrict__ rowptr,
                    const int* __restrict__ col, const int* __restrict__ seg_row,
                    const int* __restrict__ seg_begin, const int* __restrict__ seg_end,
                    int n_seg, int seg_blocks, const float* __restrict__ attn_row,
                    const float* __restrict__ attn_col, const float* __restrict__ x,
                    const float* __restrict__ pre, const float* __restrict__ emax,
                    const float* __restrict__ esum, const float* __restrict__ grad_y,
                    float slope, float p, Seed seed_in, float* __restrict__ gpre,
                    float* __restrict__ glog, float* __restrict__ grad_attn_row) {
  const uint64_t seed = seed_in;
  using V = typename VecT<VEC>::type;
  using Cfg = GatCfg<VEC, VPL, LPR>;
  const int lig = threadIdx.x % LPR;
  const int group = threadIdx.x / LPR;
  const unsigned gmask = group_mask<LPR>();

  if (static_cast<int>(blockIdx.x) < seg_blocks) {
    const int64_t sidx = static_cast<int64_t>(blockIdx.x) * Cfg::kGroups + group;
    if (sidx >= n_seg) return;
    const int64_t row = seg_row[sidx];
    const int e0 = seg_begin[sidx], e1 = seg_end[sidx];
    for (int64_t f0 = 0; f0 < C; f0 += Cfg::kTile) {
      V g[VPL];
      k1_gpre<VEC, VPL, LPR>(row, C, f0, H, lig, false, grad_y, pre, gpre, g);
      k1_dots<VEC, VPL, LPR>(e0, e1, H, C, f0, f0 == 0, col, x, g, lig, gmask, glog);
    }
    return;
  }

  const int64_t r64 = static_cast<int64_t>(blockIdx.x - seg_blocks) * Cfg::kGroups + group;
  if (r64 >= n) return;
  const int e0 = rowptr[r64], e1 = rowptr[r64 + 1];
  if (e1 - e0 > kSegLen) return;
  for (int64_t f0 = 0; f0 < C; f0 += Cfg::kTile) {
    V g[VPL];
    k1_gpre<VEC, VPL, LPR>(r64, C, f0, H, lig, true, grad_y, pre, gpre, g);
    k1_dots<VEC, VPL, LPR>(e0, e1, H, C, f0, f0 == 0, col, x, g, lig, gmask, glog);
  }
  // Each lane re-reads only the glog entries it wrote itself (same
  // lane -> edge mapping), so no synchronisation is needed.
  for (int h = 0; h < H; ++h) {
    const float ad = attn_row[r64 * H + h];
    const float m = emax[r64 * H + h], s = esum[r64 * H + h];
    float wsum = 0.0f;
    for (int e = e0 + lig; e < e1; e += LPR) {
      const EdgeSoft es = edge_soft(ad, attn_col[static_cast<int64_t>(col[e]) * H + h], m, s, slope,
                                    p, seed, static_cast<uint64_t>(e) * H + h,
                                    glog[static_cast<int64_t>(e) * H + h]);
      wsum += es.soft * es.ge;
    }
    wsum = group_sum<LPR>(wsum, gmask);
    float grow = 0.0f;
    for (int e = e0 + lig; e < e1; e += LPR) {
      const int64_t o = static_cast<int64_t>(e) * H + h;
      const EdgeSoft es = edge_soft(ad, attn_col[static_cast<int64_t>(col[e]) * H + h], m, s, slope,
                                    p, seed, static_cast<uint64_t>(e) * H + h, glog[o]);
      float gout = es.soft * (es.ge - wsum);
      if (es.neg) gout *= slope;
      glog[o] = gout;
      grow += gout;
    }
    grow = group_sum<LPR>(grow, gmask);
    if (lig == 0) grad_attn_row[r64 * H + h] = grow;
  }
}

// Hub rows, CTA (hub, head): the softmax backward of that head over the
// row's edges (dots already in glog from the segment groups); the head-0 CTA
// also writes the row's g_pre.
__global__ void __launch_bounds__(kHubThreads)
gat_bwd_hub_rows_kernel(int H, int64_t C, const int* __restrict__ rowptr,
                        const int* __restrict__ col, const int* __restrict__ hub_row,
                        const float* __restrict__ attn_row, const float* __restrict__ attn_col,
                        const float* __restrict__ pre, const float* __restrict__ emax,
                        const float* __restrict__ esum, const float* __restrict__ grad_y,
                        float slope, float p, Seed seed_in, float* __restrict__ gpre,
                        float* __restrict__ glog, float* __restrict__ grad_attn_row) {
  const uint64_t seed = seed_in;
  __shared__ float scratch[32];
  const int64_t row = hub_row[blockIdx.x];
  const int h = blockIdx.y;
  if (h == 0 && grad_y != nullptr) {
    for (int64_t c = threadIdx.x; c < C; c += kHubThreads)
      gpre[row * C + c] = grad_y[row * C + c] * silu_grad_f(pre[row * C + c]);
  }
  const int e0 = rowptr[row], e1 = rowptr[row + 1];
  const float ad = attn_row[row * H + h];
  const float m = emax[row * H + h], s = esum[row * H + h];
  // A thread's edges e0 + tid, + kHubThreads, ... in groups of kHubBatch
  // whose col / attn_col / glog loads are issued together (the largest hub
  // row of a power-law graph gives each thread a few dozen edges); the
  // per-thread sums still run over the edges in order.
  float wsum = 0.0f;
  for (int eb = e0 + threadIdx.x; eb < e1; eb += kHubBatch * kHubThreads) {
    float ac[kHubBatch], gl[kHubBatch];
#pragma unroll
    for (int u = 0; u < kHubBatch; ++u) {
      const int e = eb + u * kHubThreads;
      const int cc = e < e1 ? col[e] : 0;
      ac[u] = e < e1 ? attn_col[static_cast<int64_t>(cc) * H + h] : 0.0f;
      gl[u] = e < e1 ? glog[static_cast<int64_t>(e) * H + h] : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < kHubBatch; ++u) {
      const int e = eb + u * kHubThreads;
      if (e >= e1) break;
      const EdgeSoft es = edge_soft(ad, ac[u], m, s, slope, p, seed,
                                    static_cast<uint64_t>(e) * H + h, gl[u]);
      wsum += es.soft * es.ge;
    }
  }
  wsum = block_sum<kHubThreads>(wsum, scratch);
  float grow = 0.0f;
  for (int eb = e0 + threadIdx.x; eb < e1; eb += kHubBatch * kHubThreads) {
    float ac[kHubBatch], gl[kHubBatch];
#pragma unroll
    for (int u = 0; u < kHubBatch; ++u) {
      const int e = eb + u * kHubThreads;
      const int cc = e < e1 ? col[e] : 0;
      ac[u] = e < e1 ? attn_col[static_cast<int64_t>(cc) * H + h] : 0.0f;
      gl[u] = e < e1 ? glog[static_cast<int64_t>(e) * H + h] : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < kHubBatch; ++u) {
      const int e = eb + u * kHubThreads;
      if (e >= e1) break;
      const int64_t o = static_cast<int64_t>(e) * H + h;
      const EdgeSoft es = edge_soft(ad, ac[u], m, s, slope, p, seed,
                                    static_cast<uint64_t>(e) * H + h, gl[u]);
      float gout = es.soft * (es.ge - wsum);
      if (es.neg) gout *= slope;
      glog[o] = gout;
      grow += gout;
    }
  }
  grow = block_sum<kHubThreads>(grow, scratch);
  if (threadIdx.x == 0) grad_attn_row[row * H + h] = grow;
}

// ------------------------------------------------------------ backward K2
// acc[hh] += w(e, h0+hh) / H * g_pre[row[pos], tile] over CSC positions
// [p0, p1) of column j.
template <int VEC, int VPL, int LPR, int HB>
__device__ __forceinline__ void k2_gather(int64_t j, int p0, int p1, int H, int h0, int64_t C,
                                          int64_t f0, const int* __restrict__ row,
                                          const int* __restrict__ perm,
                                          const float* __restrict__ attn_row,
                                          const float* __restrict__ attn_col,
                                          const float* __restrict__ emax,
                                          const float* __restrict__ esum,
                                          const float* __restrict__ gpre, float slope, float p,
                                          uint64_t seed, int lig, unsigned gmask,
                                          typename VecT<VEC>::type (&acc)[HB][VPL]) {
  using V = typename VecT<VEC>::type;
  const float inv_h = 1.0f / static_cast<float>(H);
  for (int base = p0; base < p1; base += LPR) {
    const int pos = base + lig;
    const bool valid = pos < p1;
    int i = 0;
    float w[HB];
#pragma unroll
    for (int hh = 0; hh < HB; ++hh) w[hh] = 0.0f;
    if (valid) {
      i = __ldg(row + pos);
      const int e = __ldg(perm + pos);
#pragma unroll
      for (int hh = 0; hh < HB; ++hh) {
        const int h = h0 + hh;
        if (h < H) {
          const int64_t ih = static_cast<int64_t>(i) * H + h;
          w[hh] = edge_weight(__ldg(attn_row + ih), __ldg(attn_col + j * H + h), __ldg(emax + ih),
                              __ldg(esum + ih), slope, p, seed,
                              static_cast<uint64_t>(e) * H + h) * inv_h;
        }
      }
    }
    const int cnt = min(LPR, p1 - base);
    int t = 0;
    for (; t + 2 <= cnt; t += 2) {
      const int i0 = __shfl_sync(gmask, i, t, LPR);
      const int i1 = __shfl_sync(gmask, i, t + 1, LPR);
      float w0[HB], w1[HB];
#pragma unroll
      for (int hh = 0; hh < HB; ++hh) {
        w0[hh] = __shfl_sync(gmask, w[hh], t, LPR);
        w1[hh] = __shfl_sync(gmask, w[hh], t + 1, LPR);
      }
      V g0[VPL], g1[VPL];
#pragma unroll
      for (int q = 0; q < VPL; ++q) {
        const int64_t fi = static_cast<int64_t>(lig + q * LPR) * VEC;
        if (f0 + fi < C) {
          g0[q] = ldg_vec<VEC>(gpre + static_cast<int64_t>(i0) * C + f0 + fi);
          g1[q] = ldg_vec<VEC>(gpre + static_cast<int64_t>(i1) * C + f0 + fi);
        } else {
          vzero(g0[q]);
          vzero(g1[q]);
        }
      }
#pragma unroll
      for (int hh = 0; hh < HB; ++hh)
#pragma unroll
        for (int q = 0; q < VPL; ++q) {
          vfma(acc[hh][q], w0[hh], g0[q]);
          vfma(acc[hh][q], w1[hh], g1[q]);
        }
    }
    for (; t < cnt; ++t) {
      const int i0 = __shfl_sync(gmask, i, t, LPR);
      float w0[HB];
#pragma unroll
      for (int hh = 0; hh < HB; ++hh) w0[hh] = __shfl_sync(gmask, w[hh], t, LPR);
#pragma unroll
      for (int q = 0; q < VPL; ++q) {
        const int64_t fi = static_cast<int64_t>(lig + q * LPR) * VEC;
        if (f0 + fi < C) {
          const V g0 = ldg_vec<VEC>(gpre + static_cast<int64_t>(i0) * C + f0 + fi);
#pragma unroll
          for (int hh = 0; hh < HB; ++hh) vfma(acc[hh][q], w0[hh], g0);
        }
      }
    }
  }
}

// Blocks [0, seg_blocks): hub-column segments -> partial grad_feat
// [n_seg, H*C] and partial grad_attn_col [n_seg, H]; remaining blocks:
// whole columns.
template <int VEC, int VPL, int LPR, int HB>
__global__ void __launch_bounds__(kThreads)
gat_bwd_cols_kernel(int n, int H, int64_t C, const int* __restrict__ colptr,
                    const int* __restrict__ row, const int* __restrict__ perm,
                    const int* __restrict__ seg_col, const int* __restrict__ seg_begin,
                    const int* __restrict__ seg_end, int n_seg, int seg_blocks,
                    const float* __restrict__ attn_row, const float* __restrict__ attn_col,
                    const float* __restrict__ emax, const float* __restrict__ esum,
                    const float* __restrict__ gpre, const float* __restrict__ glog,
                    float slope, float p, Seed seed_in, float* __restrict__ grad_feat,
                    float* __restrict__ grad_attn_col, float* __restrict__ pfeat,
                    float* __restrict__ pcol) {
  const uint64_t seed = seed_in;
  using V = typename VecT<VEC>::type;
  using Cfg = GatCfg<VEC, VPL, LPR>;
  const int lig = threadIdx.x % LPR;
  const int group = threadIdx.x / LPR;
  const unsigned gmask = group_mask<LPR>();
  const int64_t HC = static_cast<int64_t>(H) * C;

  int64_t j64, out_idx;
  int p0, p1;
  float* fdst;
  float* cdst;
  if (static_cast<int>(blockIdx.x) < seg_blocks) {
    const int64_t sidx = static_cast<int64_t>(blockIdx.x) * Cfg::kGroups + group;
    if (sidx >= n_seg) return;
    j64 = seg_col[sidx];
    p0 = seg_begin[sidx];
    p1 = seg_end[sidx];
    out_idx = sidx;
    fdst = pfeat;
    cdst = pcol;
  } else {
    j64 = static_cast<int64_t>(blockIdx.x - seg_blocks) * Cfg::kGroups + group;
    if (j64 >= n) return;
    p0 = colptr[j64];
    p1 = colptr[j64 + 1];
    if (p1 - p0 > kSegLen) return;  // hub column: segments + combine
    out_idx = j64;
    fdst = grad_feat;
    cdst = grad_attn_col;
  }
  for (int h = 0; h < H; ++h) {
    float a = 0.0f;
    for (int pos = p0 + lig; pos < p1; pos += LPR)
      a += glog[static_cast<int64_t>(perm[pos]) * H + h];
    a = group_sum<LPR>(a, gmask);
    if (lig == 0) cdst[out_idx * H + h] = a;
  }
  for (int h0 = 0; h0 < H; h0 += HB) {
    for (int64_t f0 = 0; f0 < C; f0 += Cfg::kTile) {
      V acc[HB][VPL];
#pragma unroll
      for (int hh = 0; hh < HB; ++hh)
#pragma unroll
        for (int q = 0; q < VPL; ++q) vzero(acc[hh][q]);
      k2_gather<VEC, VPL, LPR, HB>(j64, p0, p1, H, h0, C, f0, row, perm, attn_row, attn_col, emax,
                                   esum, gpre, slope, p, seed, lig, gmask, acc);
#pragma unroll
      for (int hh = 0; hh < HB; ++hh) {
        if (h0 + hh >= H) break;
#pragma unroll
        for (int q = 0; q < VPL; ++q) {
          const int64_t fi = static_cast<int64_t>(lig + q * LPR) * VEC;
          if (f0 + fi < C)
            st_vec(fdst + out_idx * HC + static_cast<int64_t>(h0 + hh) * C + f0 + fi, acc[hh][q]);
        }
      }
    }
  }
}

// Hub-column combine: grad_feat[j] / grad_attn_col[j] = sums of the
// column's segment partials in segment order.  Block (hub, chunk) covers
// kCombineThreads * VEC of the H*C features; chunk 0 also does the H logits.
// Its kSegCombineWays thread rows each sum a contiguous share of the
// segments (the largest hub of a power-law graph has over a hundred), and
// way 0 then adds the shares in way order: a fixed order, with a critical
// path a share long instead of the whole segment list.
constexpr int kSegCombineWays = 4;
template <int VEC>
__global__ void __launch_bounds__(kCombineThreads * kSegCombineWays)
gat_bwd_cols_combine_kernel(int H, int64_t C, const int* __restrict__ hub_col,
                            const int* __restrict__ hub_first, const float* __restrict__ pfeat,
                            const float* __restrict__ pcol, float* __restrict__ grad_feat,
                            float* __restrict__ grad_attn_col) {
  using V = typename VecT<VEC>::type;
  __shared__ V part[kSegCombineWays - 1][kCombineThreads];
  __shared__ float lpart[kSegCombineWays - 1][kCombineThreads];
  const int tx = threadIdx.x % kCombineThreads, way = threadIdx.x / kCombineThreads;
  const int64_t j = hub_col[blockIdx.x];
  const int s0 = hub_first[blockIdx.x], s1 = hub_first[blockIdx.x + 1];
  const int per = (s1 - s0 + kSegCombineWays - 1) / kSegCombineWays;
  const int a = min(s1, s0 + way * per), b = min(s1, a + per);
  const int64_t HC = static_cast<int64_t>(H) * C;
  const int64_t k = (static_cast<int64_t>(blockIdx.y) * kCombineThreads + tx) * VEC;
  const bool logits = blockIdx.y == 0 && pcol != nullptr;
  V acc;
  vzero(acc);
  if (k < HC) acc = ordered_sum<VEC>(pfeat + k, HC, a, b);
  // the H logit sums (H <= kCombineThreads), in the same shares
  float lacc = 0.0f;
  if (logits && tx < H) lacc = ordered_sum<1>(pcol + tx, H, a, b);
  if (way > 0) {
    part[way - 1][tx] = acc;
    lpart[way - 1][tx] = lacc;
  }
  __syncthreads();
  if (way > 0) return;
#pragma unroll
  for (int w = 0; w < kSegCombineWays - 1; ++w) {
    vadd(acc, part[w][tx]);
    lacc += lpart[w][tx];
  }
  if (k < HC) st_vec(grad_feat + j * HC + k, acc);
  if (logits && tx < H) grad_attn_col[j * H + tx] = lacc;
}

// ------------------------------------------------------------ misc kernels
__global__ void gat_mask_kernel(int64_t total, float p, Seed seed_in,
                                uint8_t* __restrict__ mask) {
  const uint64_t seed = seed_in;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += stride)
    mask[i] = gat_keep(seed, static_cast<uint64_t>(i), p) ? 1 : 0;
}

__global__ void gat_validate_kernel(int64_t n, int64_t n_cols, int64_t nnz,
                                    const int* __restrict__ rowptr,
                                    const int* __restrict__ col, const int* __restrict__ colptr,
                                    const int* __restrict__ row, const int* __restrict__ perm,
                                    int* __restrict__ bad) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  for (int64_t i = t0; i < n; i += stride)
    if (rowptr[i] > rowptr[i + 1]) atomicOr(bad, 1);
  for (int64_t i = t0; i < n_cols; i += stride)
    if (colptr[i] > colptr[i + 1]) atomicOr(bad, 2);
  for (int64_t e = t0; e < nnz; e += stride) {
    const int c = col[e];
    if (c < 0 || c >= n_cols) atomicOr(bad, 4);
    const int r = row[e];
    if (r < 0 || r >= n) { atomicOr(bad, 8); continue; }
    const int pe = perm[e];
    if (pe < 0 || pe >= nnz) { atomicOr(bad, 16); continue; }
    // The CSR edge perm[e] must lie in row r's CSR range.
    if (pe < rowptr[r] || pe >= rowptr[r + 1]) atomicOr(bad, 32);
  }
  // CSC position pos of column j must map to a CSR edge whose column is j.
  for (int64_t j = t0; j < n_cols; j += stride) {
    const int lo = max(colptr[j], 0);
    const int hi = min(static_cast<int64_t>(colptr[j + 1]), nnz);
    for (int pos = lo; pos < hi; ++pos) {
      const int pe = perm[pos];
      if (pe >= 0 && pe < nnz && col[pe] != j) { atomicOr(bad, 64); break; }
    }
  }
  if (t0 == 0) {
    if (rowptr[0] != 0 || rowptr[n] != nnz) atomicOr(bad, 128);
    if (colptr[0] != 0 || colptr[n_cols] != nnz) atomicOr(bad, 256);
  }
}


// ====================================================================
// Persistent cp.async ring kernels (C % 4 == 0, 16-byte aligned operands,
// H <= kRingMaxH).  Work items (segments of hub rows/columns first, then
// rows/columns of at most kSegLen edges, so every item has <= 32 edges:
// one chunk) are taken from an atomic counter by whole warps.  For each
// edge the warp streams the gathered feature tiles into a warp-private ring
// of STAGES shared-memory slots with 16-byte cp.async copies, so STAGES
// edges' rows are in flight per warp without holding registers; each lane
// reads back only the float4 slots it copied itself.  The per-(edge, head)
// softmax weights of the item are computed once by the edge-owner lanes and
// kept in a warp-private shared array.  Sum orders are fixed (edge order
// within an item, segment order in the combine kernels): deterministic.
// ====================================================================
constexpr int kRingThreads = 128;
constexpr int kRingMaxH = 8;

struct RingItem {
  int64_t node;   // destination row (forward, K1) or source column (K2)
  int e0, e1;     // edge range (CSR edges, or CSC positions for K2)
  int seg;        // segment index, or -1 for a whole row/column
};

// Items [0, n_seg) are segments; [n_seg, n_seg + n) nodes.  Returns false
// for a node that is a hub (handled by its segments).
__device__ __forceinline__ bool ring_item(int it, int n_seg, const int* __restrict__ seg_node,
                                          const int* __restrict__ seg_begin,
                                          const int* __restrict__ seg_end,
                                          const int* __restrict__ ptr, RingItem& r) {
  if (it < n_seg) {
    r.node = seg_node[it];
    r.e0 = seg_begin[it];
    r.e1 = seg_end[it];
    r.seg = it;
    return true;
  }
  r.node = it - n_seg;
  r.e0 = ptr[r.node];
  r.e1 = ptr[r.node + 1];
  r.seg = -1;
  return r.e1 - r.e0 <= kSegLen;
}

__device__ __forceinline__ int ring_next(int* counter, int lane) {
  int it = 0;
  if (lane == 0) it = atomicAdd(counter, 1);
  return __shfl_sync(kFullMask, it, 0);
}

// Forward.  Items are (channel tile, item) pairs, tile-major.
template <int STAGES>
__global__ void __launch_bounds__(kRingThreads)
gat_fwd_ring_kernel(int n, int H, int64_t C, const int* __restrict__ rowptr,
                    const int* __restrict__ col, const int* __restrict__ seg_row,
                    const int* __restrict__ seg_begin, const int* __restrict__ seg_end, int n_seg,
                    const float* __restrict__ attn_row, const float* __restrict__ attn_col,
                    const float* __restrict__ x, const float* __restrict__ bias, float slope,
                    float p, Seed seed_in, float* __restrict__ out, float* __restrict__ pre,
                    float* __restrict__ emax, float* __restrict__ esum,
                    float* __restrict__ partial, int* __restrict__ counter) {
  const uint64_t seed = seed_in;
  extern __shared__ float4 smem4[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int slot_f4 = H * 32;  // one 128-channel tile of every head
  float4* ring = smem4 + warp * STAGES * slot_f4;
  float* wsm = reinterpret_cast<float*>(smem4 + (kRingThreads / 32) * STAGES * slot_f4) +
               warp * 32 * kRingMaxH;
  const int64_t HC = static_cast<int64_t>(H) * C;
  const int per_tile = n_seg + n;
  const int64_t n_tiles = (C + 127) / 128;
  const int64_t total = n_tiles * per_tile;
  const float hf = static_cast<float>(H);
  for (;;) {
    const int64_t item = ring_next(counter, lane);
    if (item >= total) break;
    const int64_t f0 = (item / per_tile) * 128;
    RingItem r;
    if (!ring_item(static_cast<int>(item % per_tile), n_seg, seg_row, seg_begin, seg_end, rowptr, r))
      continue;
    const int cnt = r.e1 - r.e0;
    const int my = r.e0 + lane;
    const int c = lane < cnt ? __ldg(col + my) : 0;
    // per-(edge, head) weights of the item
    for (int h = 0; h < H; ++h) {
      const float ad = __ldg(attn_row + r.node * H + h);
      const float ac = lane < cnt ? __ldg(attn_col + static_cast<int64_t>(c) * H + h) : 0.0f;
      float m, s;
      if (r.seg >= 0) {
        m = emax[r.node * H + h];
        s = esum[r.node * H + h];
      } else {
        const float e = lane < cnt ? leaky_f(ad + ac, slope) : kNegInit;
        m = warp_max(e);
        s = warp_sum(lane < cnt ? expf(e - m) : 0.0f);
        if (lane == 0 && f0 == 0) {
          emax[r.node * H + h] = m;
          esum[r.node * H + h] = s;
        }
      }
      wsm[lane * kRingMaxH + h] =
          lane < cnt ? edge_weight(ad, ac, m, s, slope, p, seed, static_cast<uint64_t>(my) * H + h)
                     : 0.0f;
    }
    __syncwarp();
    const bool valid = f0 + lane * 4 < C;
    const float* xt = x + f0 + lane * 4;
    auto issue = [&](int k) {
      if (k < cnt) {
        const int ck = __shfl_sync(kFullMask, c, k);
        float4* dst = ring + (k % STAGES) * slot_f4 + lane;
        const float* src = xt + static_cast<int64_t>(ck) * HC;
        if (valid)
          for (int h = 0; h < H; ++h) cp_async16(dst + h * 32, src + static_cast<int64_t>(h) * C);
      }
      cp_async_commit();
    };
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int k = 0; k < STAGES; ++k) issue(k);
    for (int k = 0; k < cnt; ++k) {
      cp_async_wait<STAGES - 1>();
      if (valid) {
        const float4* slot = ring + (k % STAGES) * slot_f4 + lane;
        for (int h = 0; h < H; ++h) vfma(acc, wsm[k * kRingMaxH + h], slot[h * 32]);
      }
      __syncwarp();
      issue(k + STAGES);
    }
    cp_async_wait<0>();
    __syncwarp();
    if (valid) {
      const int64_t fi = f0 + lane * 4;
      if (r.seg >= 0) {
        st_vec(partial + static_cast<int64_t>(r.seg) * C + fi, acc);
      } else {
        const float4 bv = ldg_vec<4>(bias + fi);
        float4 pv, ov;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float pj = vel(acc, j) / hf + vel(bv, j);
          vel(pv, j) = pj;
          vel(ov, j) = silu_f(pj);
        }
        st_vec(pre + r.node * C + fi, pv);
        st_vec(out + r.node * C + fi, ov);
      }
    }
  }
}

// Backward K1 (CSR rows): per item, per 128-channel tile, the dots of
// g_pre[i]/H with every edge's x[j, h, tile]; the edge-owner lane
// accumulates them over tiles.  Whole rows then run the softmax backward in
// the warp; segments store their dots (the hub-row kernel finishes them).
template <int STAGES>
__global__ void __launch_bounds__(kRingThreads)
gat_bwd_rows_ring_kernel(int n, int H, int64_t C, const int* __restrict__ rowptr,
                         const int* __restrict__ col, const int* __restrict__ seg_row,
                         const int* __restrict__ seg_begin, const int* __restrict__ seg_end,
                         int n_seg, const float* __restrict__ attn_row,
                         const float* __restrict__ attn_col, const float* __restrict__ x,
                         const float* __restrict__ pre, const float* __restrict__ emax,
                         const float* __restrict__ esum, const float* __restrict__ grad_y,
                         float slope, float p, Seed seed_in, float* __restrict__ gpre,
                         float* __restrict__ glog, float* __restrict__ grad_attn_row,
                         int* __restrict__ counter) {
  const uint64_t seed = seed_in;
  extern __shared__ float4 smem4[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int slot_f4 = H * 32;
  float4* ring = smem4 + warp * STAGES * slot_f4;
  const int64_t HC = static_cast<int64_t>(H) * C;
  const int total = n_seg + n;
  const float inv_h = 1.0f / static_cast<float>(H);
  for (;;) {
    const int it = ring_next(counter, lane);
    if (it >= total) break;
    RingItem r;
    if (!ring_item(it, n_seg, seg_row, seg_begin, seg_end, rowptr, r)) continue;
    const int cnt = r.e1 - r.e0;
    const int my = r.e0 + lane;
    const int c = lane < cnt ? __ldg(col + my) : 0;
    float dacc[kRingMaxH];
#pragma unroll
    for (int h = 0; h < kRingMaxH; ++h) dacc[h] = 0.0f;
    for (int64_t f0 = 0; f0 < C; f0 += 128) {
      const int64_t fi = f0 + lane * 4;
      const bool valid = fi < C;
      float4 g = make_float4(0.f, 0.f, 0.f, 0.f);
      if (valid) {
        const float4 gy = ld_vec<4>(grad_y + r.node * C + fi);
        const float4 pr = ld_vec<4>(pre + r.node * C + fi);
        float4 gp;
#pragma unroll
        for (int j = 0; j < 4; ++j) vel(gp, j) = vel(gy, j) * silu_grad_f(vel(pr, j));
        if (r.seg < 0) st_vec(gpre + r.node * C + fi, gp);
#pragma unroll
        for (int j = 0; j < 4; ++j) vel(g, j) = vel(gp, j) * inv_h;
      }
      const float* xt = x + fi;
      auto issue = [&](int k) {
        if (k < cnt) {
          const int ck = __shfl_sync(kFullMask, c, k);
          float4* dst = ring + (k % STAGES) * slot_f4 + lane;
          const float* src = xt + static_cast<int64_t>(ck) * HC;
          if (valid)
            for (int h = 0; h < H; ++h) cp_async16(dst + h * 32, src + static_cast<int64_t>(h) * C);
        }
        cp_async_commit();
      };
#pragma unroll
      for (int k = 0; k < STAGES; ++k) issue(k);
      for (int k = 0; k < cnt; ++k) {
        cp_async_wait<STAGES - 1>();
        const float4* slot = ring + (k % STAGES) * slot_f4 + lane;
#pragma unroll
        for (int h = 0; h < kRingMaxH; ++h) {
          if (h < H) {
            float d = 0.0f;
            if (valid) {
              const float4 xv = slot[h * 32];
              d = g.x * xv.x;
              d = fmaf(g.y, xv.y, d);
              d = fmaf(g.z, xv.z, d);
              d = fmaf(g.w, xv.w, d);
            }
            d = warp_sum(d);
            if (lane == k) dacc[h] += d;
          }
        }
        __syncwarp();
        issue(k + STAGES);
      }
      cp_async_wait<0>();
      __syncwarp();
    }
    if (r.seg >= 0) {
      if (lane < cnt) {
#pragma unroll
        for (int h = 0; h < kRingMaxH; ++h)
          if (h < H) glog[static_cast<int64_t>(my) * H + h] = dacc[h];
      }
      continue;
    }
#pragma unroll
    for (int h = 0; h < kRingMaxH; ++h) {
      if (h >= H) break;
      const float ad = attn_row[r.node * H + h];
      const float m = emax[r.node * H + h], s = esum[r.node * H + h];
      EdgeSoft es;
      es.soft = 0.0f;
      es.ge = 0.0f;
      es.neg = false;
      if (lane < cnt)
        es = edge_soft(ad, attn_col[static_cast<int64_t>(c) * H + h], m, s, slope, p, seed,
                       static_cast<uint64_t>(my) * H + h, dacc[h]);
      const float wsum = warp_sum(es.soft * es.ge);
      float gout = es.soft * (es.ge - wsum);
      if (es.neg) gout *= slope;
      if (lane < cnt) glog[static_cast<int64_t>(my) * H + h] = gout;
      const float grow = warp_sum(lane < cnt ? gout : 0.0f);
      if (lane == 0) grad_attn_row[r.node * H + h] = grow;
    }
  }
}

// Backward K2 (CSC columns): items are (256-channel tile, item) pairs,
// tile-major.  grad_feat[j,h,tile] = sum_e w(e,h)/H g_pre[i_e, tile];
// grad_attn_col[j,h] = sum_e grad_logit[e,h] (tile 0 only).
template <int STAGES>
__global__ void __launch_bounds__(kRingThreads)
gat_bwd_cols_ring_kernel(int n, int H, int64_t C, const int* __restrict__ colptr,
                         const int* __restrict__ row, const int* __restrict__ perm,
                         const int* __restrict__ seg_col, const int* __restrict__ seg_begin,
                         const int* __restrict__ seg_end, int n_seg,
                         const float* __restrict__ attn_row, const float* __restrict__ attn_col,
                         const float* __restrict__ emax, const float* __restrict__ esum,
                         const float* __restrict__ gpre, const float* __restrict__ glog,
                         float slope, float p, Seed seed_in, float* __restrict__ grad_feat,
                         float* __restrict__ grad_attn_col, float* __restrict__ pfeat,
                         float* __restrict__ pcol, int* __restrict__ counter) {
  const uint64_t seed = seed_in;
  constexpr int VPL = 2;
  extern __shared__ float4 smem4[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int kSlot = 32 * VPL;
  float4* ring = smem4 + warp * STAGES * kSlot;
  float* wsm = reinterpret_cast<float*>(smem4 + (kRingThreads / 32) * STAGES * kSlot) +
               warp * 32 * kRingMaxH;
  const int64_t HC = static_cast<int64_t>(H) * C;
  const int per_tile = n_seg + n;
  const int64_t n_tiles = (C + 4 * kSlot - 1) / (4 * kSlot);
  const int64_t total = n_tiles * per_tile;
  const float inv_h = 1.0f / static_cast<float>(H);
  for (;;) {
    const int64_t item = ring_next(counter, lane);
    if (item >= total) break;
    const int64_t f0 = (item / per_tile) * (4 * kSlot);
    RingItem r;
    if (!ring_item(static_cast<int>(item % per_tile), n_seg, seg_col, seg_begin, seg_end, colptr, r))
      continue;
    const int cnt = r.e1 - r.e0;
    const int pos = r.e0 + lane;
    int i = 0, e = 0;
    if (lane < cnt) {
      i = __ldg(row + pos);
      e = __ldg(perm + pos);
    }
    for (int h = 0; h < H; ++h) {
      float w = 0.0f;
      if (lane < cnt) {
        const int64_t ih = static_cast<int64_t>(i) * H + h;
        w = edge_weight(__ldg(attn_row + ih), __ldg(attn_col + r.node * H + h), __ldg(emax + ih),
                        __ldg(esum + ih), slope, p, seed, static_cast<uint64_t>(e) * H + h) * inv_h;
      }
      wsm[lane * kRingMaxH + h] = w;
      if (f0 == 0) {
        const float a = warp_sum(lane < cnt ? glog[static_cast<int64_t>(e) * H + h] : 0.0f);
        if (lane == 0) {
          if (r.seg >= 0) pcol[static_cast<int64_t>(r.seg) * H + h] = a;
          else grad_attn_col[r.node * H + h] = a;
        }
      }
    }
    __syncwarp();
    const float* gt = gpre + f0 + lane * 4;
    auto issue = [&](int k) {
      if (k < cnt) {
        const int ik = __shfl_sync(kFullMask, i, k);
        float4* dst = ring + (k % STAGES) * kSlot + lane;
        const float* src = gt + static_cast<int64_t>(ik) * C;
#pragma unroll
        for (int q = 0; q < VPL; ++q)
          if (f0 + (lane + q * 32) * 4 < C) cp_async16(dst + q * 32, src + q * 128);
      }
      cp_async_commit();
    };
    float4 acc[kRingMaxH][VPL];
#pragma unroll
    for (int h = 0; h < kRingMaxH; ++h)
#pragma unroll
      for (int q = 0; q < VPL; ++q) acc[h][q] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int k = 0; k < STAGES; ++k) issue(k);
    for (int k = 0; k < cnt; ++k) {
      cp_async_wait<STAGES - 1>();
      const float4* slot = ring + (k % STAGES) * kSlot + lane;
#pragma unroll
      for (int q = 0; q < VPL; ++q) {
        if (f0 + (lane + q * 32) * 4 < C) {
          const float4 gv = slot[q * 32];
#pragma unroll
          for (int h = 0; h < kRingMaxH; ++h)
            if (h < H) vfma(acc[h][q], wsm[k * kRingMaxH + h], gv);
        }
      }
      __syncwarp();
      issue(k + STAGES);
    }
    cp_async_wait<0>();
    __syncwarp();
    float* dst = r.seg >= 0 ? pfeat + static_cast<int64_t>(r.seg) * HC : grad_feat + r.node * HC;
#pragma unroll
    for (int h = 0; h < kRingMaxH; ++h) {
      if (h >= H) break;
#pragma unroll
      for (int q = 0; q < VPL; ++q) {
        const int64_t fi = f0 + (lane + q * 32) * 4;
        if (fi < C) st_vec(dst + static_cast<int64_t>(h) * C + fi, acc[h][q]);
      }
    }
  }
}

constexpr int kFwdStages = 6;
constexpr int kK1Stages = 6;
constexpr int kK2Stages = 8;

// The kernel's dynamic shared-memory limit is raised to its largest use
// (H = kRingMaxH) once; the persistent grid is sized for the actual use.
template <typename K>
int ring_grid(K kernel, size_t smem, size_t max_smem, int* cache) {
  if (*cache == 0) {
    CIGN_CHECK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(max_smem)),
                    "gat: set smem");
    *cache = persistent_grid(kernel, kRingThreads, smem);
  }
  return CIGN_OK;
}

size_t fwd_ring_smem(int H) {
  return static_cast<size_t>(kRingThreads / 32) *
         (static_cast<size_t>(kFwdStages) * H * 32 * 16 + 32 * kRingMaxH * sizeof(float));
}
size_t k1_ring_smem(int H) {
  return static_cast<size_t>(kRingThreads / 32) * kK1Stages * H * 32 * 16;
}
size_t k2_ring_smem() {
  return static_cast<size_t>(kRingThreads / 32) *
         (static_cast<size_t>(kK2Stages) * 2 * 32 * 16 + 32 * kRingMaxH * sizeof(float));
}

// ------------------------------------------------------------ hub launches
int launch_hub_stats(const cign_gat_plan* pl, int H, const float* attn_row, const float* attn_col,
                     float slope, float* emax, float* esum, cudaStream_t s) {
  const SegList& sl = pl->rows;
  if (sl.n_heavy == 0) return CIGN_OK;
  gat_hub_stats_kernel<<<dim3(static_cast<unsigned>(sl.n_heavy), H), kHubThreads, 0, s>>>(
      H, pl->rowptr, pl->col, sl.heavy_row(), attn_row, attn_col, slope, emax, esum);
  CIGN_CHECK_LAUNCH("gat_hub_stats_kernel");
  return CIGN_OK;
}

// Vector width of the combine kernels: 4 when every operand allows float4.
bool combine_v4(int64_t n_feat, std::initializer_list<const void*> ptrs) {
  if (n_feat % 4 != 0) return false;
  for (const void* q : ptrs)
    if (!aligned16(q)) return false;
  return true;
}

unsigned combine_chunks(int64_t n_feat, int vec) {
  const int64_t per_block = static_cast<int64_t>(kCombineThreads) * vec;
  return static_cast<unsigned>((n_feat + per_block - 1) / per_block);
}

int launch_fwd_combine(const cign_gat_plan* pl, int H, int64_t C, const float* partial,
                       const float* bias, float* pre, float* out, cudaStream_t s) {
  const SegList& sl = pl->rows;
  if (sl.n_heavy == 0) return CIGN_OK;
  const bool v4 = combine_v4(C, {partial, bias, pre, out});
  const dim3 grid(static_cast<unsigned>(sl.n_heavy), combine_chunks(C, v4 ? 4 : 1));
  CIGN_REQUIRE(grid.y < 65536, CIGN_ERR_UNSUPPORTED, "gat: C too large for the hub combine");
  if (v4)
    gat_fwd_combine_kernel<4><<<grid, kCombineThreads, 0, s>>>(H, C, sl.heavy_row(),
                                                               sl.heavy_first(), partial, bias, pre,
                                                               out);
  else
    gat_fwd_combine_kernel<1><<<grid, kCombineThreads, 0, s>>>(H, C, sl.heavy_row(),
                                                               sl.heavy_first(), partial, bias, pre,
                                                               out);
  CIGN_CHECK_LAUNCH("gat_fwd_combine_kernel");
  return CIGN_OK;
}

int launch_bwd_hub_rows(const cign_gat_plan* pl, int H, int64_t C, const float* attn_row,
                        const float* attn_col, const float* pre, const float* emax,
                        const float* esum, const float* gy, float slope, float p, Seed seed,
                        float* gpre, float* glog, float* grow, cudaStream_t s) {
  const SegList& sl = pl->rows;
  if (sl.n_heavy == 0) return CIGN_OK;
  gat_bwd_hub_rows_kernel<<<dim3(static_cast<unsigned>(sl.n_heavy), H), kHubThreads, 0, s>>>(
      H, C, pl->rowptr, pl->col, sl.heavy_row(), attn_row, attn_col, pre, emax, esum, gy, slope,
      p, seed, gpre, glog, grow);
  CIGN_CHECK_LAUNCH("gat_bwd_hub_rows_kernel");
  return CIGN_OK;
}

int launch_seg_combine(const SegList& sl, int H, int64_t C, const float* pfeat, const float* pcol,
                       float* gfeat, float* gcol, cudaStream_t s);

int launch_bwd_cols_combine(const cign_gat_plan* pl, int H, int64_t C, const float* pfeat,
                            const float* pcol, float* gfeat, float* gcol, cudaStream_t s) {
  return launch_seg_combine(pl->cols, H, C, pfeat, pcol, gfeat, gcol, s);
}

// out[target] = ordered sum of the target's segment partials ([n_seg, H*C]),
// and, when pcol is not NULL, gcol[target] = the same over pcol ([n_seg, H]).
int launch_seg_combine(const SegList& sl, int H, int64_t C, const float* pfeat, const float* pcol,
                       float* gfeat, float* gcol, cudaStream_t s) {
  if (sl.n_heavy == 0) return CIGN_OK;
  const int64_t HC = static_cast<int64_t>(H) * C;
  const bool v4 = combine_v4(HC, {pfeat, gfeat});
  const dim3 grid(static_cast<unsigned>(sl.n_heavy), combine_chunks(HC, v4 ? 4 : 1));
  CIGN_REQUIRE(grid.y < 65536, CIGN_ERR_UNSUPPORTED, "gat: H*C too large for the hub combine");
  CIGN_REQUIRE(pcol == nullptr || H <= kCombineThreads, CIGN_ERR_UNSUPPORTED,
               "gat: too many heads for the hub combine");
  if (v4)
    gat_bwd_cols_combine_kernel<4><<<grid, kCombineThreads * kSegCombineWays, 0, s>>>(
        H, C, sl.heavy_row(), sl.heavy_first(), pfeat, pcol, gfeat, gcol);
  else
    gat_bwd_cols_combine_kernel<1><<<grid, kCombineThreads * kSegCombineWays, 0, s>>>(
        H, C, sl.heavy_row(), sl.heavy_first(), pfeat, pcol, gfeat, gcol);
  CIGN_CHECK_LAUNCH("gat_bwd_cols_combine_kernel");
  return CIGN_OK;
}

int launch_fwd_ring(const cign_gat_plan* pl, int H, int64_t C, const float* attn_row,
                    const float* attn_col, const float* x, const float* bias, float slope,
                    float p, Seed seed, float* out, float* pre, float* emax, float* esum,
                    float* partial, int* counter, cudaStream_t s) {
  const SegList& sl = pl->rows;
  {
    const int rc = launch_hub_stats(pl, H, attn_row, attn_col, slope, emax, esum, s);
    if (rc) return rc;
  }
  static thread_local int cache[64][kRingMaxH + 1] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  auto kernel = gat_fwd_ring_kernel<kFwdStages>;
  const size_t smem = fwd_ring_smem(H);
  int rc = ring_grid(kernel, smem, fwd_ring_smem(kRingMaxH), &cache[dev & 63][H]);
  if (rc) return rc;
  CIGN_CHECK_CUDA(cudaMemsetAsync(counter, 0, sizeof(int), s), "gat: reset counter");
  kernel<<<cache[dev & 63][H], kRingThreads, smem, s>>>(
      static_cast<int>(pl->n), H, C, pl->rowptr, pl->col, sl.seg_row(), sl.seg_begin(),
      sl.seg_end(), static_cast<int>(sl.n_seg), attn_row, attn_col, x, bias, slope, p, seed, out,
      pre, emax, esum, partial, counter);
  CIGN_CHECK_LAUNCH("gat_fwd_ring_kernel");
  return launch_fwd_combine(pl, H, C, partial, bias, pre, out, s);
}

int launch_bwd_rows_ring(const cign_gat_plan* pl, int H, int64_t C, const float* attn_row,
                         const float* attn_col, const float* x, const float* pre,
                         const float* emax, const float* esum, const float* gy, float slope,
                         float p, Seed seed, float* gpre, float* glog, float* grow,
                         int* counter, cudaStream_t s) {
  const SegList& sl = pl->rows;
  static thread_local int cache[64][kRingMaxH + 1] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  auto kernel = gat_bwd_rows_ring_kernel<kK1Stages>;
  const size_t smem = k1_ring_smem(H);
  int rc = ring_grid(kernel, smem, k1_ring_smem(kRingMaxH), &cache[dev & 63][H]);
  if (rc) return rc;
  CIGN_CHECK_CUDA(cudaMemsetAsync(counter, 0, sizeof(int), s), "gat: reset counter");
  kernel<<<cache[dev & 63][H], kRingThreads, smem, s>>>(
      static_cast<int>(pl->n), H, C, pl->rowptr, pl->col, sl.seg_row(), sl.seg_begin(),
      sl.seg_end(), static_cast<int>(sl.n_seg), attn_row, attn_col, x, pre, emax, esum, gy, slope,
      p, seed, gpre, glog, grow, counter);
  CIGN_CHECK_LAUNCH("gat_bwd_rows_ring_kernel");
  {
    const int rc = launch_bwd_hub_rows(pl, H, C, attn_row, attn_col, pre, emax, esum, gy, slope, p,
                                       seed, gpre, glog, grow, s);
    if (rc) return rc;
  }
  return CIGN_OK;
}

int launch_bwd_cols_ring(const cign_gat_plan* pl, int H, int64_t C, const float* attn_row,
                         const float* attn_col, const float* emax, const float* esum,
                         const float* gpre, const float* glog, float slope, float p,
                         Seed seed, float* gfeat, float* gcol, float* pfeat, float* pcol,
                         int* counter, cudaStream_t s) {
  const SegList& sl = pl->cols;
  static thread_local int cache[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  auto kernel = gat_bwd_cols_ring_kernel<kK2Stages>;
  const size_t smem = k2_ring_smem();
  int rc = ring_grid(kernel, smem, smem, &cache[dev & 63]);
  if (rc) return rc;
  CIGN_CHECK_CUDA(cudaMemsetAsync(counter, 0, sizeof(int), s), "gat: reset counter");
  kernel<<<cache[dev & 63], kRingThreads, smem, s>>>(
      static_cast<int>(pl->n_cols), H, C, pl->colptr, pl->row, pl->perm, sl.seg_row(), sl.seg_begin(),
      sl.seg_end(), static_cast<int>(sl.n_seg), attn_row, attn_col, emax, esum, gpre, glog, slope,
      p, seed, gfeat, gcol, pfeat, pcol, counter);
  CIGN_CHECK_LAUNCH("gat_bwd_cols_ring_kernel");
  return launch_bwd_cols_combine(pl, H, C, pfeat, pcol, gfeat, gcol, s);
}


// ====================================================================
// TMA-ring kernels (C % 4 == 0, 16-byte aligned operands, H <= kRingMaxH,
// gathered row <= kTmaSlotMax bytes).  Same work items as the cp.async ring
// kernels (every item has <= 32 edges), but each gathered row -- the whole
// [H, C] block of x[j] in the forward and K1, the C-wide g_pre[i] row in K2
// -- is ONE cp.async.bulk copy issued by lane 0 and completed on its slot's
// mbarrier.  Waits are bounded; on expiry the warp records kStatusTimeout in
// ctl[1], lets its in-flight copies land (bounded) and stops.
// ====================================================================
constexpr int kTmaWarps = 4;
constexpr uint32_t kTmaSlotMax = 16384;

struct TmaWarpRing {
  float* slots;
  uint64_t* bars;
  float* wsm;
  int stages;
  int slot_floats;
  uint32_t phase;
};

// smem layout: [slots of all warps][barriers of all warps][weights of all warps]
__device__ __forceinline__ TmaWarpRing tma_ring_setup(unsigned char* smem, int stages,
                                                      int slot_floats, int warp, int lane) {
  TmaWarpRing r;
  r.stages = stages;
  r.slot_floats = slot_floats;
  r.phase = 0;
  const size_t slot_bytes_all = static_cast<size_t>(kTmaWarps) * stages * slot_floats * 4;
  r.slots = reinterpret_cast<float*>(smem) + static_cast<size_t>(warp) * stages * slot_floats;
  r.bars = reinterpret_cast<uint64_t*>(smem + slot_bytes_all) + warp * stages;
  r.wsm = reinterpret_cast<float*>(smem + slot_bytes_all + kTmaWarps * stages * 8) +
          warp * 32 * kRingMaxH;
  if (lane == 0) {
    for (int s = 0; s < stages; ++s) mbar_init(smem_u32(&r.bars[s]), 1);
    fence_mbar_init();
  }
  __syncwarp();
  return r;
}
size_t tma_smem_bytes(int stages, int slot_floats) {
  return static_cast<size_t>(kTmaWarps) *
         (static_cast<size_t>(stages) * (slot_floats * 4 + 8) + 32 * kRingMaxH * 4);
}
int tma_stages(uint32_t slot_bytes, int target_bytes, int lo, int hi) {
  return std::max(lo, std::min(hi, static_cast<int>(target_bytes / slot_bytes)));
}

// lane 0: arm slot k % stages and copy `bytes` from src into it
__device__ __forceinline__ void tma_fill(TmaWarpRing& r, int k, const float* src, uint32_t bytes,
                                         int lane) {
  if (lane == 0) {
    const int sl = k % r.stages;
    const uint32_t bar = smem_u32(&r.bars[sl]);
    mbar_expect_tx(bar, bytes);
    bulk_g2s(smem_u32(r.slots + static_cast<size_t>(sl) * r.slot_floats), src, bytes, bar);
  }
}
// all lanes: wait for slot k % stages; false (warp-uniform) on timeout
__device__ __forceinline__ bool tma_take(TmaWarpRing& r, int k) {
  const int sl = k % r.stages;
  const bool got = mbar_wait(smem_u32(&r.bars[sl]), (r.phase >> sl) & 1u);
  if (!__all_sync(kFullMask, got)) return false;
  r.phase ^= 1u << sl;
  return true;
}
// after the warp consumed slot k % stages: order its reads before a refill
__device__ __forceinline__ void tma_release(int lane) {
  __syncwarp();
  if (lane == 0) fence_proxy_async();
}
// on failure: let fills [lo, hi) land (bounded) before the warp stops
__device__ __forceinline__ void tma_drain(TmaWarpRing& r, int lo, int hi, int* status, int lane) {
  if (lane == 0) atomicExch(status, kStatusTimeout);
  for (int k = lo; k < hi; ++k) {
    const int sl = k % r.stages;
    mbar_wait(smem_u32(&r.bars[sl]), (r.phase >> sl) & 1u);
    r.phase ^= 1u << sl;
  }
}

// Forward: items are whole rows / hub segments.
template <int VPL>
__global__ void __launch_bounds__(kTmaWarps * 32)
gat_fwd_tma_kernel(int n, int H, int64_t C, const int* __restrict__ rowptr,
                   const int* __restrict__ col, const int* __restrict__ seg_row,
                   const int* __restrict__ seg_begin, const int* __restrict__ seg_end, int n_seg,
                   const float* __restrict__ attn_row, const float* __restrict__ attn_col,
                   const float* __restrict__ x, const float* __restrict__ bias, float slope,
                   float p, Seed seed_in, float* __restrict__ out, float* __restrict__ pre,
                   float* __restrict__ emax, float* __restrict__ esum,
                   float* __restrict__ partial, int stages, int* __restrict__ ctl) {
  const uint64_t seed = seed_in;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t HC = static_cast<int64_t>(H) * C;
  TmaWarpRing ring = tma_ring_setup(smem_raw, stages, static_cast<int>(HC), warp, lane);
  const uint32_t bytes = static_cast<uint32_t>(HC * 4);
  const int C4 = static_cast<int>(C / 4);
  const int total = n_seg + n;
  const float hf = static_cast<float>(H);
  for (;;) {
    const int it = ring_next(ctl, lane);
    if (it >= total) break;
    RingItem r;
    if (!ring_item(it, n_seg, seg_row, seg_begin, seg_end, rowptr, r)) continue;
    const int cnt = r.e1 - r.e0;
    const int my = r.e0 + lane;
    const int c = lane < cnt ? __ldg(col + my) : 0;
    auto issue = [&](int k) {
      if (k < cnt) {
        const int ck = __shfl_sync(kFullMask, c, k);
        tma_fill(ring, k, x + static_cast<int64_t>(ck) * HC, bytes, lane);
      }
    };
    for (int k = 0; k < stages; ++k) issue(k);  // copies overlap the weight math
    for (int h = 0; h < H; ++h) {
      const float ad = __ldg(attn_row + r.node * H + h);
      const float ac = lane < cnt ? __ldg(attn_col + static_cast<int64_t>(c) * H + h) : 0.0f;
      float m, sm;
      if (r.seg >= 0) {
        m = emax[r.node * H + h];
        sm = esum[r.node * H + h];
      } else {
        const float e = lane < cnt ? leaky_f(ad + ac, slope) : kNegInit;
        m = warp_max(e);
        sm = warp_sum(lane < cnt ? expf(e - m) : 0.0f);
        if (lane == 0) {
          emax[r.node * H + h] = m;
          esum[r.node * H + h] = sm;
        }
      }
      ring.wsm[lane * kRingMaxH + h] =
          lane < cnt ? edge_weight(ad, ac, m, sm, slope, p, seed, static_cast<uint64_t>(my) * H + h)
                     : 0.0f;
    }
    __syncwarp();
    float4 acc[VPL];
#pragma unroll
    for (int q = 0; q < VPL; ++q) acc[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < cnt; ++k) {
      if (!tma_take(ring, k)) {
        tma_drain(ring, k, min(k + stages, cnt), ctl + 1, lane);
        return;
      }
      const float4* slot = reinterpret_cast<const float4*>(ring.slots + static_cast<size_t>(k % stages) * HC);
      for (int h = 0; h < H; ++h) {
        const float w = ring.wsm[k * kRingMaxH + h];
#pragma unroll
        for (int q = 0; q < VPL; ++q)
          if (lane + q * 32 < C4) vfma(acc[q], w, slot[h * C4 + lane + q * 32]);
      }
      tma_release(lane);
      issue(k + stages);
    }
#pragma unroll
    for (int q = 0; q < VPL; ++q) {
      if (lane + q * 32 >= C4) continue;
      const int64_t fi = static_cast<int64_t>(lane + q * 32) * 4;
      if (r.seg >= 0) {
        st_vec(partial + static_cast<int64_t>(r.seg) * C + fi, acc[q]);
      } else {
        const float4 bv = ldg_vec<4>(bias + fi);
        float4 pv, ov;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float pj = vel(acc[q], j) / hf + vel(bv, j);
          vel(pv, j) = pj;
          vel(ov, j) = silu_f(pj);
        }
        st_vec(pre + r.node * C + fi, pv);
        st_vec(out + r.node * C + fi, ov);
      }
    }
  }
}

// Backward K1 (CSR rows) on the TMA ring: dots of g_pre[i]/H with each
// edge's x[j] block, then the softmax backward (whole rows) or the dots
// stored for the hub-row kernel (segments).
template <int VPL>
__global__ void __launch_bounds__(kTmaWarps * 32)
gat_bwd_rows_tma_kernel(int n, int H, int64_t C, const int* __restrict__ rowptr,
                        const int* __restrict__ col, const int* __restrict__ seg_row,
                        const int* __restrict__ seg_begin, const int* __restrict__ seg_end,
                        int n_seg, const float* __restrict__ attn_row,
                        const float* __restrict__ attn_col, const float* __restrict__ x,
                        const float* __restrict__ pre, const float* __restrict__ emax,
                        const float* __restrict__ esum, const float* __restrict__ grad_y,
                        float slope, float p, Seed seed_in, float* __restrict__ gpre,
                        float* __restrict__ glog, float* __restrict__ grad_attn_row,
                        int stages, int* __restrict__ ctl) {
  const uint64_t seed = seed_in;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t HC = static_cast<int64_t>(H) * C;
  TmaWarpRing ring = tma_ring_setup(smem_raw, stages, static_cast<int>(HC), warp, lane);
  const uint32_t bytes = static_cast<uint32_t>(HC * 4);
  const int C4 = static_cast<int>(C / 4);
  const int total = n_seg + n;
  const float inv_h = 1.0f / static_cast<float>(H);
  for (;;) {
    const int it = ring_next(ctl, lane);
    if (it >= total) break;
    RingItem r;
    if (!ring_item(it, n_seg, seg_row, seg_begin, seg_end, rowptr, r)) continue;
    const int cnt = r.e1 - r.e0;
    const int my = r.e0 + lane;
    const int c = lane < cnt ? __ldg(col + my) : 0;
    auto issue = [&](int k) {
      if (k < cnt) {
        const int ck = __shfl_sync(kFullMask, c, k);
        tma_fill(ring, k, x + static_cast<int64_t>(ck) * HC, bytes, lane);
      }
    };
    for (int k = 0; k < stages; ++k) issue(k);
    float4 g[VPL];
#pragma unroll
    for (int q = 0; q < VPL; ++q) {
      g[q] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (lane + q * 32 < C4) {
        const int64_t fi = static_cast<int64_t>(lane + q * 32) * 4;
        const float4 gy = ld_vec<4>(grad_y + r.node * C + fi);
        const float4 pr = ld_vec<4>(pre + r.node * C + fi);
        float4 gp;
#pragma unroll
        for (int j = 0; j < 4; ++j) vel(gp, j) = vel(gy, j) * silu_grad_f(vel(pr, j));
        if (r.seg < 0) st_vec(gpre + r.node * C + fi, gp);
#pragma unroll
        for (int j = 0; j < 4; ++j) vel(g[q], j) = vel(gp, j) * inv_h;
      }
    }
    float dacc[kRingMaxH];
#pragma unroll
    for (int h = 0; h < kRingMaxH; ++h) dacc[h] = 0.0f;
    for (int k = 0; k < cnt; ++k) {
      if (!tma_take(ring, k)) {
        tma_drain(ring, k, min(k + stages, cnt), ctl + 1, lane);
        return;
      }
      const float4* slot = reinterpret_cast<const float4*>(ring.slots + static_cast<size_t>(k % stages) * HC);
#pragma unroll
      for (int h = 0; h < kRingMaxH; ++h) {
        if (h < H) {
          float d = 0.0f;
#pragma unroll
          for (int q = 0; q < VPL; ++q) {
            if (lane + q * 32 < C4) {
              const float4 xv = slot[h * C4 + lane + q * 32];
              d = fmaf(g[q].x, xv.x, d);
              d = fmaf(g[q].y, xv.y, d);
              d = fmaf(g[q].z, xv.z, d);
              d = fmaf(g[q].w, xv.w, d);
            }
          }
          d = warp_sum(d);
          if (lane == k) dacc[h] = d;
        }
      }
      tma_release(lane);
      issue(k + stages);
    }
    if (r.seg >= 0) {
      if (lane < cnt) {
#pragma unroll
        for (int h = 0; h < kRingMaxH; ++h)
          if (h < H) glog[static_cast<int64_t>(my) * H + h] = dacc[h];
      }
      continue;
    }
#pragma unroll
    for (int h = 0; h < kRingMaxH; ++h) {
      if (h >= H) break;
      const float ad = attn_row[r.node * H + h];
      const float m = emax[r.node * H + h], s = esum[r.node * H + h];
      EdgeSoft es;
      es.soft = 0.0f;
      es.ge = 0.0f;
      es.neg = false;
      if (lane < cnt)
        es = edge_soft(ad, attn_col[static_cast<int64_t>(c) * H + h], m, s, slope, p, seed,
                       static_cast<uint64_t>(my) * H + h, dacc[h]);
      const float wsum = warp_sum(es.soft * es.ge);
      float gout = es.soft * (es.ge - wsum);
      if (es.neg) gout *= slope;
      if (lane < cnt) glog[static_cast<int64_t>(my) * H + h] = gout;
      const float grow = warp_sum(lane < cnt ? gout : 0.0f);
      if (lane == 0) grad_attn_row[r.node * H + h] = grow;
    }
  }
}

// Backward K2 (CSC columns) on the TMA ring: g_pre[i] rows, heads in groups
// of four accumulated in registers.
template <int VPL>
__global__ void __launch_bounds__(kTmaWarps * 32)
gat_bwd_cols_tma_kernel(int n, int H, int64_t C, const int* __restrict__ colptr,
                        const int* __restrict__ row, const int* __restrict__ perm,
                        const int* __restrict__ seg_col, const int* __restrict__ seg_begin,
                        const int* __restrict__ seg_end, int n_seg,
                        const float* __restrict__ attn_row, const float* __restrict__ attn_col,
                        const float* __restrict__ emax, const float* __restrict__ esum,
                        const float* __restrict__ gpre, const float* __restrict__ glog,
                        float slope, float p, Seed seed_in, float* __restrict__ grad_feat,
                        float* __restrict__ grad_attn_col, float* __restrict__ pfeat,
                        float* __restrict__ pcol, int stages, int* __restrict__ ctl) {
  const uint64_t seed = seed_in;
  constexpr int HB = 4;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  TmaWarpRing ring = tma_ring_setup(smem_raw, stages, static_cast<int>(C), warp, lane);
  const uint32_t bytes = static_cast<uint32_t>(C * 4);
  const int C4 = static_cast<int>(C / 4);
  const int64_t HC = static_cast<int64_t>(H) * C;
  const int total = n_seg + n;
  const float inv_h = 1.0f / static_cast<float>(H);
  for (;;) {
    const int it = ring_next(ctl, lane);
    if (it >= total) break;
    RingItem r;
    if (!ring_item(it, n_seg, seg_col, seg_begin, seg_end, colptr, r)) continue;
    const int cnt = r.e1 - r.e0;
    const int pos = r.e0 + lane;
    int i = 0, e = 0;
    if (lane < cnt) {
      i = __ldg(row + pos);
      e = __ldg(perm + pos);
    }
    for (int h = 0; h < H; ++h) {
      float w = 0.0f;
      if (lane < cnt) {
        const int64_t ih = static_cast<int64_t>(i) * H + h;
        w = edge_weight(__ldg(attn_row + ih), __ldg(attn_col + r.node * H + h), __ldg(emax + ih),
                        __ldg(esum + ih), slope, p, seed, static_cast<uint64_t>(e) * H + h) * inv_h;
      }
      ring.wsm[lane * kRingMaxH + h] = w;
      const float a = warp_sum(lane < cnt ? glog[static_cast<int64_t>(e) * H + h] : 0.0f);
      if (lane == 0) {
        if (r.seg >= 0) pcol[static_cast<int64_t>(r.seg) * H + h] = a;
        else grad_attn_col[r.node * H + h] = a;
      }
    }
    __syncwarp();
    float* dst = r.seg >= 0 ? pfeat + static_cast<int64_t>(r.seg) * HC : grad_feat + r.node * HC;
    auto issue = [&](int k) {
      if (k < cnt) {
        const int ik = __shfl_sync(kFullMask, i, k);
        tma_fill(ring, k, gpre + static_cast<int64_t>(ik) * C, bytes, lane);
      }
    };
    for (int h0 = 0; h0 < H; h0 += HB) {
      float4 acc[HB][VPL];
#pragma unroll
      for (int hh = 0; hh < HB; ++hh)
#pragma unroll
        for (int q = 0; q < VPL; ++q) acc[hh][q] = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int k = 0; k < stages; ++k) issue(k);
      for (int k = 0; k < cnt; ++k) {
        if (!tma_take(ring, k)) {
          tma_drain(ring, k, min(k + stages, cnt), ctl + 1, lane);
          return;
        }
        const float4* slot = reinterpret_cast<const float4*>(ring.slots + static_cast<size_t>(k % stages) * C);
#pragma unroll
        for (int q = 0; q < VPL; ++q) {
          if (lane + q * 32 < C4) {
            const float4 gv = slot[lane + q * 32];
#pragma unroll
            for (int hh = 0; hh < HB; ++hh)
              if (h0 + hh < H) vfma(acc[hh][q], ring.wsm[k * kRingMaxH + h0 + hh], gv);
          }
        }
        tma_release(lane);
        issue(k + stages);
      }
#pragma unroll
      for (int hh = 0; hh < HB; ++hh) {
        if (h0 + hh >= H) break;
#pragma unroll
        for (int q = 0; q < VPL; ++q)
          if (lane + q * 32 < C4)
            st_vec(dst + static_cast<int64_t>(h0 + hh) * C + static_cast<int64_t>(lane + q * 32) * 4,
                   acc[hh][q]);
      }
    }
  }
}

// Persistent grid for `kernel` with `smem` bytes, cached per (device, smem);
// the kernel's dynamic shared-memory limit is raised once per device.
template <typename K>
int tma_grid(K kernel, size_t smem, int* grid) {
  static std::mutex mu;
  static std::map<std::pair<int, size_t>, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find({dev, smem});
  if (it != cache.end()) {
    *grid = it->second;
    return CIGN_OK;
  }
  CIGN_CHECK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       227 * 1024),
                  "gat: set smem");
  *grid = persistent_grid(kernel, kTmaWarps * 32, smem);
  cache[{dev, smem}] = *grid;
  return CIGN_OK;
}

#define CIGN_TMA_VPL_DISPATCH(C4_, CALL)                        \
  do {                                                          \
    if ((C4_) <= 32) { constexpr int P_ = 1; CALL; }            \
    else if ((C4_) <= 64) { constexpr int P_ = 2; CALL; }       \
    else if ((C4_) <= 128) { constexpr int P_ = 4; CALL; }      \
    else { constexpr int P_ = 8; CALL; }                        \
  } while (0)

template <int VPL>
int launch_fwd_tma_vpl(const cign_gat_plan* pl, int H, int64_t C, const float* attn_row,
                       const float* attn_col, const float* x, const float* bias, float slope,
                       float p, Seed seed, float* out, float* pre, float* emax, float* esum,
                       float* partial, int* ctl, cudaStream_t s) {
  const SegList& sl = pl->rows;
  {
    const int rc = launch_hub_stats(pl, H, attn_row, attn_col, slope, emax, esum, s);
    if (rc) return rc;
  }
  const uint32_t slot_bytes = static_cast<uint32_t>(H * C * 4);
  const int stages = tma_stages(slot_bytes, 24576, 2, 8);
  const size_t smem = tma_smem_bytes(stages, static_cast<int>(H * C));
  auto kernel = gat_fwd_tma_kernel<VPL>;
  int grid = 0;
  int rc = tma_grid(kernel, smem, &grid);
  if (rc) return rc;
  CIGN_CHECK_CUDA(cudaMemsetAsync(ctl, 0, 2 * sizeof(int), s), "gat: reset control");
  kernel<<<grid, kTmaWarps * 32, smem, s>>>(
      static_cast<int>(pl->n), H, C, pl->rowptr, pl->col, sl.seg_row(), sl.seg_begin(),
      sl.seg_end(), static_cast<int>(sl.n_seg), attn_row, attn_col, x, bias, slope, p, seed, out,
      pre, emax, esum, partial, stages, ctl);
  CIGN_CHECK_LAUNCH("gat_fwd_tma_kernel");
  return launch_fwd_combine(pl, H, C, partial, bias, pre, out, s);
}

template <int VPL>
int launch_bwd_rows_tma_vpl(const cign_gat_plan* pl, int H, int64_t C, const float* attn_row,
                            const float* attn_col, const float* x, const float* pre,
                            const float* emax, const float* esum, const float* gy, float slope,
                            float p, Seed seed, float* gpre, float* glog, float* grow,
                            int* ctl, cudaStream_t s) {
  const SegList& sl = pl->rows;
  const uint32_t slot_bytes = static_cast<uint32_t>(H * C * 4);
  const int stages = tma_stages(slot_bytes, 24576, 2, 8);
  const size_t smem = tma_smem_bytes(stages, static_cast<int>(H * C));
  auto kernel = gat_bwd_rows_tma_kernel<VPL>;
  int grid = 0;
  int rc = tma_grid(kernel, smem, &grid);
  if (rc) return rc;
  CIGN_CHECK_CUDA(cudaMemsetAsync(ctl, 0, 2 * sizeof(int), s), "gat: reset control");
  kernel<<<grid, kTmaWarps * 32, smem, s>>>(
      static_cast<int>(pl->n), H, C, pl->rowptr, pl->col, sl.seg_row(), sl.seg_begin(),
      sl.seg_end(), static_cast<int>(sl.n_seg), attn_row, attn_col, x, pre, emax, esum, gy, slope,
      p, seed, gpre, glog, grow, stages, ctl);
  CIGN_CHECK_LAUNCH("gat_bwd_rows_tma_kernel");
  {
    const int rc = launch_bwd_hub_rows(pl, H, C, attn_row, attn_col, pre, emax, esum, gy, slope, p,
                                       seed, gpre, glog, grow, s);
    if (rc) return rc;
  }
  return CIGN_OK;
}

template <int VPL>
int launch_bwd_cols_tma_vpl(const cign_gat_plan* pl, int H, int64_t C, const float* attn_row,
                            const float* attn_col, const float* emax, const float* esum,
                            const float* gpre, const float* glog, float slope, float p,
                            Seed seed, float* gfeat, float* gcol, float* pfeat, float* pcol,
                            int* ctl, cudaStream_t s) {
  const SegList& sl = pl->cols;
  const uint32_t slot_bytes = static_cast<uint32_t>(C * 4);
  const int stages = tma_stages(slot_bytes, 16384, 4, 8);
  const size_t smem = tma_smem_bytes(stages, static_cast<int>(C));
  auto kernel = gat_bwd_cols_tma_kernel<VPL>;
  int grid = 0;
  int rc = tma_grid(kernel, smem, &grid);
  if (rc) return rc;
  CIGN_CHECK_CUDA(cudaMemsetAsync(ctl, 0, 2 * sizeof(int), s), "gat: reset control");
  kernel<<<grid, kTmaWarps * 32, smem, s>>>(
      static_cast<int>(pl->n_cols), H, C, pl->colptr, pl->row, pl->perm, sl.seg_row(), sl.seg_begin(),
      sl.seg_end(), static_cast<int>(sl.n_seg), attn_row, attn_col, emax, esum, gpre, glog, slope,
      p, seed, gfeat, gcol, pfeat, pcol, stages, ctl);
  CIGN_CHECK_LAUNCH("gat_bwd_cols_tma_kernel");
  return launch_bwd_cols_combine(pl, H, C, pfeat, pcol, gfeat, gcol, s);
}

// ------------------------------------------------------------ dispatch
size_t rnd(size_t b) { return (b + 255) / 256 * 256; }

template <int VEC, int VPL, int LPR>
int launch_fwd_cfg(const cign_gat_plan* pl, int H, int64_t C, const float* attn_row,
                   const float* attn_col, const float* x, const float* bias, float slope, float p,
                   Seed seed, float* out, float* pre, float* emax, float* esum, float* partial,
                   cudaStream_t s) {
  using Cfg = GatCfg<VEC, VPL, LPR>;
  const SegList& sl = pl->rows;
  {
    const int rc = launch_hub_stats(pl, H, attn_row, attn_col, slope, emax, esum, s);
    if (rc) return rc;
  }
  const int64_t seg_blocks = (sl.n_seg + Cfg::kGroups - 1) / Cfg::kGroups;
  const int64_t grid = seg_blocks + (pl->n + Cfg::kGroups - 1) / Cfg::kGroups;
  const size_t smem = static_cast<size_t>(Cfg::kGroups) * 2 * H * sizeof(float);
  gat_fwd_kernel<VEC, VPL, LPR><<<static_cast<unsigned>(grid), kThreads, smem, s>>>(
      static_cast<int>(pl->n), H, C, pl->rowptr, pl->col, sl.seg_row(), sl.seg_begin(),
      sl.seg_end(), static_cast<int>(sl.n_seg), static_cast<int>(seg_blocks), attn_row, attn_col,
      x, bias, slope, p, seed, out, pre, emax, esum, partial);
  CIGN_CHECK_LAUNCH("gat_fwd_kernel");
  return launch_fwd_combine(pl, H, C, partial, bias, pre, out, s);
}

template <int VEC, int VPL, int LPR>
int launch_bwd_rows_cfg(const cign_gat_plan* pl, int H, int64_t C, const float* attn_row,
                        const float* attn_col, const float* x, const float* pre,
                        const float* emax, const float* esum, const float* gy, float slope,
                        float p, Seed seed, float* gpre, float* glog, float* grow,
                        cudaStream_t s) {
  using Cfg = GatCfg<VEC, VPL, LPR>;
  const SegList& sl = pl->rows;
  const int64_t seg_blocks = (sl.n_seg + Cfg::kGroups - 1) / Cfg::kGroups;
  const int64_t grid = seg_blocks + (pl->n + Cfg::kGroups - 1) / Cfg::kGroups;
  gat_bwd_rows_kernel<VEC, VPL, LPR><<<static_cast<unsigned>(grid), kThreads, 0, s>>>(
      static_cast<int>(pl->n), H, C, pl->rowptr, pl->col, sl.seg_row(), sl.seg_begin(),
      sl.seg_end(), static_cast<int>(sl.n_seg), static_cast<int>(seg_blocks), attn_row, attn_col,
      x, pre, emax, esum, gy, slope, p, seed, gpre, glog, grow);
  CIGN_CHECK_LAUNCH("gat_bwd_rows_kernel");
  {
    const int rc = launch_bwd_hub_rows(pl, H, C, attn_row, attn_col, pre, emax, esum, gy, slope, p,
                                       seed, gpre, glog, grow, s);
    if (rc) return rc;
  }
  return CIGN_OK;
}

template <int VEC, int VPL, int LPR, int HB>
int launch_bwd_cols_cfg(const cign_gat_plan* pl, int H, int64_t C, const float* attn_row,
                        const float* attn_col, const float* emax, const float* esum,
                        const float* gpre, const float* glog, float slope, float p, Seed seed,
                        float* gfeat, float* gcol, float* pfeat, float* pcol, cudaStream_t s) {
  using Cfg = GatCfg<VEC, VPL, LPR>;
  const SegList& sl = pl->cols;
  const int64_t seg_blocks = (sl.n_seg + Cfg::kGroups - 1) / Cfg::kGroups;
  const int64_t grid = seg_blocks + (pl->n_cols + Cfg::kGroups - 1) / Cfg::kGroups;
  gat_bwd_cols_kernel<VEC, VPL, LPR, HB><<<static_cast<unsigned>(grid), kThreads, 0, s>>>(
      static_cast<int>(pl->n_cols), H, C, pl->colptr, pl->row, pl->perm, sl.seg_row(), sl.seg_begin(),
      sl.seg_end(), static_cast<int>(sl.n_seg), static_cast<int>(seg_blocks), attn_row, attn_col,
      emax, esum, gpre, glog, slope, p, seed, gfeat, gcol, pfeat, pcol);
  CIGN_CHECK_LAUNCH("gat_bwd_cols_kernel");
  return launch_bwd_cols_combine(pl, H, C, pfeat, pcol, gfeat, gcol, s);
}

// Shape rule shared by the kernels: VEC=4 when C%4==0 and the feature
// pointers are 16-byte aligned; LPR/VPL from the number of vectors per row.
#define CIGN_GAT_DISPATCH(VEC_, FV_, CALL)                                     \
  do {                                                                         \
    if ((FV_) <= 8) { constexpr int V_ = VEC_, P_ = 1, L_ = 8; CALL; }         \
    else if ((FV_) <= 16) { constexpr int V_ = VEC_, P_ = 1, L_ = 16; CALL; }  \
    else if ((FV_) <= 32) { constexpr int V_ = VEC_, P_ = 1, L_ = 32; CALL; }  \
    else if ((FV_) <= 64) { constexpr int V_ = VEC_, P_ = 2, L_ = 32; CALL; }  \
    else if ((FV_) <= 128) { constexpr int V_ = VEC_, P_ = 4, L_ = 32; CALL; } \
    else { constexpr int V_ = VEC_, P_ = 8, L_ = 32; CALL; }                   \
  } while (0)

int check_plan(const cign_gat_plan* pl, int H, int64_t C, const char* name) {
  CIGN_REQUIRE(pl != nullptr, CIGN_ERR_NULL_POINTER, "%s: plan is NULL", name);
  CIGN_REQUIRE(H >= 1 && H <= kMaxHeads, CIGN_ERR_UNSUPPORTED,
               "%s: heads must be in [1, %d], got %d", name, kMaxHeads, H);
  CIGN_REQUIRE(C >= 1 && C < (1ll << 24), CIGN_ERR_INVALID_ARGUMENT,
               "%s: channels must be in [1, 2^24), got %lld", name, (long long)C);
  return CIGN_OK;
}

// forward workspace: hub-row partials [n_seg_rows * C] | work counter
size_t fwd_ws_bytes(const cign_gat_plan* pl, int64_t C) {
  return rnd(static_cast<size_t>(pl->rows.n_seg) * C * sizeof(float)) + 256;
}

// backward workspace: g_pre [N*C] | grad_logit [nnz*H] | colsum partials |
// column-segment partials [n_seg*(H*C)] | [n_seg*H]
struct BwdLayout {
  size_t gpre, glog, csum, pfeat, pcol, counters, total;
};
BwdLayout bwd_layout(const cign_gat_plan* pl, int H, int64_t C) {
  BwdLayout L;
  L.gpre = 0;
  L.glog = L.gpre + rnd(static_cast<size_t>(pl->n) * C * sizeof(float));
  L.csum = L.glog + rnd(static_cast<size_t>(pl->nnz) * H * sizeof(float));
  L.pfeat = L.csum + rnd(static_cast<size_t>(colsum_chunks(pl->n)) * C * sizeof(float));
  L.pcol = L.pfeat + rnd(static_cast<size_t>(pl->cols.n_seg) * H * C * sizeof(float));
  L.counters = L.pcol + rnd(static_cast<size_t>(pl->cols.n_seg) * H * sizeof(float));
  L.total = L.counters + 256;
  return L;
}

// ------------------------------------------------------ aggregate-first form
// GATConv's lin is linear, so per destination row i and head h
//   sum_j w_ijh * (W_h X_j) = W_h (sum_j w_ijh X_j).
// The aggregate-first kernels gather the layer input X [N, D] (one D-float
// row per edge, shared by all heads) instead of lin's output [N, H, C], and
// leave W to one dense GEMM afterwards:
//   forward   Z[i,h,:] = sum_j w_ijh X[j,:]                  (gat_agg_kernel, CSR)
//   backward  dots(e,h) = U[i,h,:] . X[j,:], U = dL/dZ        (gat_agg_dots_kernel, CSR)
//             grad_feat[j,h,:] = sum_i w_ijh g_pre[i,:] / H   (gat_agg_kernel, CSC)
// with the same weights w (logits, LeakyReLU, segment softmax, dropout
// stream idx = e*H + h) as the collapsed kernels above.  Every work item --
// a row (column) of at most kSegLen edges or one kSegLen-edge segment of a
// hub -- is one warp whose lane k owns edge k, so per-edge quantities are
// computed once per lane and broadcast with shuffles; feature tiles of
// 128*VPL floats run over the grid's second dimension.

constexpr int kAggHB = 4;      // heads per pass over a work item's edges
// edges per work item of the aggregation kernels: rows (columns) of up to
// this many edges are one item, longer ones are cut into items of this
// length whose partials a combine sums.  Longer items than the 32 of the
// other GAT kernels leave fewer hub partials ([items, H, D] written and read
// back) on power-law graphs.
constexpr int kAggSegLen = 128;
constexpr int kDotsSlots = 8;  // edges in the backward-K1 ring (two 4-edge groups)
constexpr size_t kDotsSmem = static_cast<size_t>(kThreads / 32) * kDotsSlots * 2 * 32 * 16;
constexpr int kAggStages = 4;  // neighbour rows in flight per warp (cp.async ring)

template <int VPL>
struct AggCfg {
  static constexpr int kGroups = kThreads / 32;  // one warp per work item
  static constexpr int kTile = 128 * VPL;        // floats per feature tile
  // dynamic shared memory: per warp, kAggStages slots of one tile, then per
  // warp the kAggHB head weights of the current chunk's 32 edges (one float4
  // per edge, read back as a broadcast)
  static constexpr size_t kRing = static_cast<size_t>(kGroups) * kAggStages * kTile * 4;
  static constexpr size_t kSmem = kRing + static_cast<size_t>(kGroups) * 32 * 16;
};

// Edge weights w[e, h] of the aggregate-first form (edge id e in CSR order),
// computed once per edge and head and read by the aggregation kernels for
// every feature tile.  Work items as in gat_agg_kernel's forward (one warp
// per row of at most kSegLen edges or per hub-row segment, lane k = edge k).
// STATS (forward): light rows compute their per-head max / exp-sum here with
// the warp reductions and write emax / esum; hub-row segments read them
// (gat_hub_stats_kernel ran first).  !STATS (backward): every row reads the
// forward's emax / esum.  The weights equal the ones the aggregation used to
// form inline, bit for bit (same reductions, same edge_weight).
template <bool STATS>
__global__ void __launch_bounds__(kThreads)
gat_edge_weights_kernel(int n_light, const int* __restrict__ light, int H,
                        const int* __restrict__ rowptr, const int* __restrict__ col,
                        const int* __restrict__ seg_row, const int* __restrict__ seg_begin,
                        const int* __restrict__ seg_end, int n_seg, int seg_blocks,
                        const float* __restrict__ attn_row, const float* __restrict__ attn_col,
                        float* __restrict__ emax, float* __restrict__ esum, float slope, float p,
                        Seed seed_in, float* __restrict__ wts) {
  const uint64_t seed = seed_in;
  const int lane = threadIdx.x & 31;
  const int group = threadIdx.x >> 5;
  int64_t target;
  int e0, e1;
  bool seg;
  if (static_cast<int>(blockIdx.x) < seg_blocks) {
    const int64_t item = static_cast<int64_t>(blockIdx.x) * (kThreads / 32) + group;
    if (item >= n_seg) return;
    target = seg_row[item];
    e0 = seg_begin[item];
    e1 = seg_end[item];
    seg = true;
  } else {  // light rows in the plan's length order
    const int64_t li = static_cast<int64_t>(blockIdx.x - seg_blocks) * (kThreads / 32) + group;
    if (li >= n_light) return;
    target = light[li];
    e0 = rowptr[target];
    e1 = rowptr[target + 1];
    seg = false;
  }
  const int k = e0 + lane;
  const bool valid = k < e1;
  const int other = valid ? __ldg(col + k) : 0;
  // kAggHB heads per pass, their reductions interleaved (each head's butterfly
  // is the one group_max / group_sum runs, so the values are the same)
  for (int h0 = 0; h0 < H; h0 += kAggHB) {
    float ad[kAggHB], lg[kAggHB], m[kAggHB], sm[kAggHB];
#pragma unroll
    for (int hh = 0; hh < kAggHB; ++hh) {
      const int h = h0 + hh < H ? h0 + hh : H - 1;
      ad[hh] = __ldg(attn_row + target * H + h);
      const float ac = valid ? __ldg(attn_col + static_cast<int64_t>(other) * H + h) : 0.0f;
      lg[hh] = leaky_f(ad[hh] + ac, slope);
    }
    if (seg || !STATS) {
#pragma unroll
      for (int hh = 0; hh < kAggHB; ++hh) {
        const int h = h0 + hh < H ? h0 + hh : H - 1;
        m[hh] = emax[target * H + h];
        sm[hh] = esum[target * H + h];
      }
    } else {
#pragma unroll
      for (int hh = 0; hh < kAggHB; ++hh) m[hh] = valid ? fmaxf(kNegInit, lg[hh]) : kNegInit;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int hh = 0; hh < kAggHB; ++hh)
          m[hh] = fmaxf(m[hh], __shfl_xor_sync(kFullMask, m[hh], o, 32));
#pragma unroll
      for (int hh = 0; hh < kAggHB; ++hh) sm[hh] = valid ? expf(lg[hh] - m[hh]) : 0.0f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int hh = 0; hh < kAggHB; ++hh) sm[hh] += __shfl_xor_sync(kFullMask, sm[hh], o, 32);
      if (lane == 0) {
#pragma unroll
        for (int hh = 0; hh < kAggHB; ++hh) {
          if (h0 + hh >= H) break;
          emax[target * H + h0 + hh] = m[hh];
          esum[target * H + h0 + hh] = sm[hh];
        }
      }
    }
    if (valid) {
#pragma unroll
      for (int hh = 0; hh < kAggHB; ++hh) {
        const int h = h0 + hh;
        if (h >= H) break;
        const uint64_t idx = static_cast<uint64_t>(k) * H + h;
        const bool keep = (p <= 0.0f) || gat_keep(seed, idx, p);
        float w = 0.0f;
        if (keep && sm[hh] > 0.0f) {  // edge_weight's expression
          w = expf(lg[hh] - m[hh]) / sm[hh];
          if (p > 0.0f) w /= (1.0f - p);
        }
        wts[static_cast<int64_t>(k) * H + h] = w;
      }
    }
  }
}

// MODE 0 (forward, CSR rows of `ptr`/`idx`): out = Z [N, H, D] from X = src;
//   hub-row segments write partials [n_seg, H, D].
// MODE 1 (backward K2, CSC columns: ptr = colptr, idx = row, perm):
//   out = grad_feat [N, H, D] from src = g_pre [N, D], scaled by 1/H; the
//   y == 0 tile also sums glog over the column into gcol (hub segments:
//   into pcol).
// Both read the edge weights from wts [nnz, H] (gat_edge_weights_kernel),
// indexed by the CSR edge id (perm[k] for a CSC position k).
// The neighbour rows are gathered by cp.async into a lane-private ring of
// kAggStages shared-memory slots per warp: lane l copies, and later reads,
// only its own 16-byte slices, so no warp synchronisation is needed, and
// kAggStages rows are in flight without occupying registers (the 4-head
// accumulator tile does).  The first copies are issued before the edge
// weights are computed, so the weight arithmetic overlaps the gather.
// Measured at cfg2 (D=512, H=4): forward 194 us against 217 us for the same
// gather from registers (two rows in flight), K2 185 us against 251 us.
template <int VPL, int MODE, bool ONE_PASS>
// <= 64 registers (1024 threads of 64 registers per SM):
__global__ void __launch_bounds__(kThreads, ONE_PASS ? 1024 / kThreads : 1)
gat_agg_kernel(int n_light, const int* __restrict__ light, int H, int64_t D,
               const int* __restrict__ ptr, const int* __restrict__ idx,
               const int* __restrict__ perm, const int* __restrict__ seg_row,
               const int* __restrict__ seg_begin, const int* __restrict__ seg_end, int n_seg,
               int seg_blocks, const float* __restrict__ wts, const float* __restrict__ src,
               float* __restrict__ out, float* __restrict__ partial,
               const float* __restrict__ glog, float* __restrict__ gcol,
               float* __restrict__ pcol) {
  extern __shared__ float4 agg_ring[];
  using Cfg = AggCfg<VPL>;
  const int lane = threadIdx.x & 31;
  const int group = threadIdx.x >> 5;
  const int64_t f0 = static_cast<int64_t>(blockIdx.y) * Cfg::kTile;
  // shared address of this lane's slot q of ring stage s:
  // agg_ring[((group * S + s) * VPL + q) * 32 + lane]
  const uint32_t my_ring =
      smem_u32(agg_ring) + static_cast<uint32_t>((group * kAggStages * VPL * 32 + lane) * 16);
  static_assert(kAggHB == 4, "one float4 of head weights per edge");
  float4* const wsm = agg_ring + Cfg::kRing / 16 + group * 32;  // this warp's weights
  int64_t item, target;
  int e0, e1;
  bool seg;
  if (static_cast<int>(blockIdx.x) < seg_blocks) {
    item = static_cast<int64_t>(blockIdx.x) * Cfg::kGroups + group;
    if (item >= n_seg) return;
    target = seg_row[item];
    e0 = seg_begin[item];
    e1 = seg_end[item];
    seg = true;
  } else {  // light rows (columns) in the plan's length order
    const int64_t li = static_cast<int64_t>(blockIdx.x - seg_blocks) * Cfg::kGroups + group;
    if (li >= n_light) return;
    target = light[li];
    e0 = ptr[target];
    e1 = ptr[target + 1];
    item = target;
    seg = false;
  }
  // this lane's feature offsets in the tile (lanes past D copy and store nothing)
  int64_t foff[VPL];
  bool fin[VPL];
#pragma unroll
  for (int q = 0; q < VPL; ++q) {
    foff[q] = f0 + static_cast<int64_t>(lane + q * 32) * 4;
    fin[q] = foff[q] < D;
  }
  const float scale = MODE == 1 ? 1.0f / static_cast<float>(H) : 1.0f;
  const int64_t HD = static_cast<int64_t>(H) * D;
  // the item's output row and (MODE 1) logit-gradient slots, fixed before
  // the edge loop so that no item bookkeeping stays live across it
  float* const dst = seg ? partial + item * HD : out + target * HD;
  float* const gdst = MODE == 1 ? (seg ? pcol + item * H : gcol + target * H) : nullptr;
  // ONE_PASS (H <= kAggHB): a single head pass with h0 = 0 known to the compiler
  for (int h0 = 0; h0 < (ONE_PASS ? 1 : H); h0 += kAggHB) {
    float4 acc[kAggHB][VPL];
#pragma unroll
    for (int hh = 0; hh < kAggHB; ++hh)
#pragma unroll
      for (int q = 0; q < VPL; ++q) acc[hh][q] = make_float4(0.f, 0.f, 0.f, 0.f);
    // MODE 1: the item's logit-gradient sum of head h0 + lane (lanes < kAggHB),
    // accumulated chunk by chunk
    float gs = 0.0f;
    // the item's edges in chunks of 32 (lane k owns edge c0 + k of a chunk)
    for (int c0 = e0; c0 < e1; c0 += 32) {
      const int k = c0 + lane;
      const bool valid = k < e1;
      const int cnt = min(32, e1 - c0);
      int other = 0;  // MODE 0: source column j; MODE 1: destination row i
      int64_t e = k;  // CSR edge id (dropout index)
      if (valid) {
        other = __ldg(idx + k);
        if (MODE == 1) e = __ldg(perm + k);
      }
      // copies of chunk edge t's tile slices into ring stage `stage`
      auto issue = [&](int t, int stage) {
        const float* xr = src + static_cast<int64_t>(__shfl_sync(kFullMask, other, t)) * D;
        const uint32_t slot = my_ring + static_cast<uint32_t>(stage * VPL * 32 * 16);
#pragma unroll
        for (int q = 0; q < VPL; ++q)
          if (fin[q]) cp_async16_s(slot + q * 32 * 16, xr + foff[q]);
      };
#pragma unroll
      for (int t = 0; t < kAggStages; ++t) {
        if (t < cnt) issue(t, t);
        cp_async_commit();
      }
      float w[kAggHB];
#pragma unroll
      for (int hh = 0; hh < kAggHB; ++hh) {
        const int h = h0 + hh;
        w[hh] = 0.0f;
        if (h >= H) continue;
        if (valid) w[hh] = __ldg(wts + e * H + h) * scale;
        if (MODE == 1 && blockIdx.y == 0) {
          const float t = group_sum<32>(valid ? glog[e * H + h] : 0.0f, kFullMask);
          if (lane == hh) gs += t;
        }
      }
      // lane k's head weights, broadcast to the warp from shared memory (one
      // 16-byte read per edge instead of kAggHB shuffles)
      wsm[lane] = make_float4(w[0], w[1], w[2], w[3]);
      __syncwarp();
      // chunk edge t sits in ring stage t % kAggStages: the loop runs
      // kAggStages edges per pass so that every stage's shared address is a
      // constant
      for (int t0 = 0; t0 < cnt; t0 += kAggStages) {
#pragma unroll
        for (int u = 0; u < kAggStages; ++u) {
          const int t = t0 + u;
          if (t >= cnt) break;
          cp_async_wait<kAggStages - 1>();  // edge t's copies have landed
          const uint32_t slot = my_ring + static_cast<uint32_t>(u * VPL * 32 * 16);
          float4 xv[VPL];
#pragma unroll
          for (int q = 0; q < VPL; ++q) xv[q] = lds_f4(slot + q * 32 * 16);
          const float4 wt = wsm[t];
#pragma unroll
          for (int hh = 0; hh < kAggHB; ++hh) {
            const float wv = vel(wt, hh);
#pragma unroll
            for (int q = 0; q < VPL; ++q) vfma(acc[hh][q], wv, xv[q]);
          }
          if (t + kAggStages < cnt) issue(t + kAggStages, u);  // into the stage just read
          cp_async_commit();
        }
      }
      cp_async_wait<0>();  // the ring is reused by the next chunk
      __syncwarp();        // and the weights
    }
    if (MODE == 1 && blockIdx.y == 0 && lane < kAggHB && h0 + lane < H) gdst[h0 + lane] = gs;
#pragma unroll
    for (int hh = 0; hh < kAggHB; ++hh) {
      if (h0 + hh >= H) break;
#pragma unroll
      for (int q = 0; q < VPL; ++q)
        if (fin[q]) st_vec(dst + static_cast<int64_t>(h0 + hh) * D + foff[q], acc[hh][q]);
    }
  }
}

// Forward aggregation over bf16 layer inputs (storage precision of the
// large-graph configuration): Z [N, H, D] fp32 = sum_j w_ijh x_j with x
// stored as bf16 and widened to fp32 as it is used; weights, edge order and
// fp32 FMA order as gat_agg_kernel<.., 0, ..>, so Z equals that kernel's
// result on the widened inputs.  Lane l copies 16 bytes = 8 bf16 per ring
// slot; a tile is 32 * VPL * 8 features.
template <int VPL>
__global__ void __launch_bounds__(kThreads)
gat_agg_fwd_bf16_kernel(int n_light, const int* __restrict__ light, int H, int64_t D,
                        const int* __restrict__ ptr, const int* __restrict__ idx,
                        const int* __restrict__ seg_row, const int* __restrict__ seg_begin,
                        const int* __restrict__ seg_end, int n_seg, int seg_blocks,
                        const float* __restrict__ attn_row, const float* __restrict__ attn_col,
                        float* __restrict__ emax, float* __restrict__ esum,
                        const __nv_bfloat16* __restrict__ src, float slope, float p,
                        Seed seed_in, float* __restrict__ out, float* __restrict__ partial) {
  extern __shared__ uint4 aggb_ring[];
  const uint64_t seed = seed_in;
  constexpr int kTile = 32 * VPL * 8;
  const int lane = threadIdx.x & 31;
  const int group = threadIdx.x >> 5;
  const int64_t f0 = static_cast<int64_t>(blockIdx.y) * kTile;
  const uint32_t my_ring =
      smem_u32(aggb_ring) + static_cast<uint32_t>((group * kAggStages * VPL * 32 + lane) * 16);
  int64_t item, target;
  int e0, e1;
  bool seg;
  if (static_cast<int>(blockIdx.x) < seg_blocks) {
    item = static_cast<int64_t>(blockIdx.x) * (kThreads / 32) + group;
    if (item >= n_seg) return;
    target = seg_row[item];
    e0 = seg_begin[item];
    e1 = seg_end[item];
    seg = true;
  } else {  // light rows in the plan's length order
    const int64_t li = static_cast<int64_t>(blockIdx.x - seg_blocks) * (kThreads / 32) + group;
    if (li >= n_light) return;
    target = light[li];
    e0 = ptr[target];
    e1 = ptr[target + 1];
    item = target;
    seg = false;
  }
  // rows of at most 32 edges form their max / exp-sum here (warp
  // reductions, as gat_edge_weights_kernel<true> does); longer rows read the
  // hub statistics (gat_hub_stats_kernel ran first)
  const bool own_stats = !seg && e1 - e0 <= 32;
  const int64_t HD = static_cast<int64_t>(H) * D;
  float* const dst = seg ? partial + item * HD : out + target * HD;
  for (int h0 = 0; h0 < H; h0 += kAggHB) {
    float acc[kAggHB][VPL][8];
#pragma unroll
    for (int hh = 0; hh < kAggHB; ++hh)
#pragma unroll
      for (int q = 0; q < VPL; ++q)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[hh][q][j] = 0.0f;
    // the item's edges in chunks of 32 (lane k owns edge c0 + k of a chunk)
    for (int c0 = e0; c0 < e1; c0 += 32) {
      const int k = c0 + lane;
      const bool valid = k < e1;
      const int cnt = min(32, e1 - c0);
      const int other = valid ? __ldg(idx + k) : 0;
      auto issue = [&](int t) {
        const __nv_bfloat16* xr =
            src + static_cast<int64_t>(__shfl_sync(kFullMask, other, t)) * D;
        const uint32_t slot = my_ring + static_cast<uint32_t>((t % kAggStages) * VPL * 32 * 16);
#pragma unroll
        for (int q = 0; q < VPL; ++q) {
          const int64_t fi = f0 + static_cast<int64_t>(lane + q * 32) * 8;
          if (fi < D) cp_async16_s(slot + q * 32 * 16, xr + fi);
        }
      };
#pragma unroll
      for (int t = 0; t < kAggStages; ++t) {
        if (t < cnt) issue(t);
        cp_async_commit();
      }
      float w[kAggHB];
#pragma unroll
      for (int hh = 0; hh < kAggHB; ++hh) {
        const int h = h0 + hh;
        w[hh] = 0.0f;
        if (h >= H) continue;
        const float ad = __ldg(attn_row + target * H + h);
        const float ac = valid ? __ldg(attn_col + static_cast<int64_t>(other) * H + h) : 0.0f;
        float m, ssum;
        if (!own_stats) {
          m = emax[target * H + h];
          ssum = esum[target * H + h];
        } else {
          m = group_max<32>(valid ? fmaxf(kNegInit, leaky_f(ad + ac, slope)) : kNegInit,
                            kFullMask);
          ssum = group_sum<32>(valid ? expf(leaky_f(ad + ac, slope) - m) : 0.0f, kFullMask);
          if (blockIdx.y == 0 && lane == 0) {
            emax[target * H + h] = m;
            esum[target * H + h] = ssum;
          }
        }
        if (valid)
          w[hh] = edge_weight(ad, ac, m, ssum, slope, p, seed, static_cast<uint64_t>(k) * H + h);
      }
      for (int t = 0; t < cnt; ++t) {
        cp_async_wait<kAggStages - 1>();
        const uint32_t slot = my_ring + static_cast<uint32_t>((t % kAggStages) * VPL * 32 * 16);
        float xf[VPL][8];
#pragma unroll
        for (int q = 0; q < VPL; ++q) {
          const float4 raw = lds_f4(slot + q * 32 * 16);
          const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f2 = __bfloat1622float2(b[i]);
            xf[q][2 * i] = f2.x;
            xf[q][2 * i + 1] = f2.y;
          }
        }
#pragma unroll
        for (int hh = 0; hh < kAggHB; ++hh) {
          const float wv = __shfl_sync(kFullMask, w[hh], t);
#pragma unroll
          for (int q = 0; q < VPL; ++q)
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[hh][q][j] = fmaf(wv, xf[q][j], acc[hh][q][j]);
        }
        if (t + kAggStages < cnt) issue(t + kAggStages);
        cp_async_commit();
      }
      cp_async_wait<0>();  // the ring is reused by the next chunk
    }
#pragma unroll
    for (int hh = 0; hh < kAggHB; ++hh) {
      if (h0 + hh >= H) break;
#pragma unroll
      for (int q = 0; q < VPL; ++q) {
        const int64_t fi = f0 + static_cast<int64_t>(lane + q * 32) * 8;
        if (fi >= D) continue;
        float* o = dst + static_cast<int64_t>(h0 + hh) * D + fi;
        st_vec(o, make_float4(acc[hh][q][0], acc[hh][q][1], acc[hh][q][2], acc[hh][q][3]));
        st_vec(o + 4, make_float4(acc[hh][q][4], acc[hh][q][5], acc[hh][q][6], acc[hh][q][7]));
      }
    }
  }
}

// Backward K1 of the aggregate-first form (CSR rows): dots(e,h) =
// U[i,h,:] . X[j,:] over D in 256-float chunks (the row's U chunk in
// registers, the neighbour's X chunk loaded once for all heads), reduced
// across the warp; the lane owning edge e keeps its dots.  Light rows then
// run the softmax/dropout/LeakyReLU backward in registers and write glog and
// grad_attn_row; hub segments write their dots to glog for the hub-row kernel.
// <= 80 registers (768 threads of 80 registers per SM):
__global__ void __launch_bounds__(kThreads, 768 / kThreads)
gat_agg_dots_kernel(int n_light, const int* __restrict__ light, int H, int64_t D,
                    const int* __restrict__ rowptr,
                    const int* __restrict__ col, const int* __restrict__ seg_row,
                    const int* __restrict__ seg_begin, const int* __restrict__ seg_end, int n_seg,
                    int seg_blocks, const float* __restrict__ attn_row,
                    const float* __restrict__ attn_col, const float* __restrict__ emax,
                    const float* __restrict__ esum, const float* __restrict__ U,
                    const float* __restrict__ X, float slope, float p, Seed seed_in,
                    float* __restrict__ glog, float* __restrict__ grad_attn_row) {
  extern __shared__ float4 dots_ring[];
  const uint64_t seed = seed_in;
  constexpr int kChunk = 256;  // floats of D per pass: 2 float4 per lane
  const int lane = threadIdx.x & 31;
  const int group = threadIdx.x >> 5;
  // lane-private ring of kDotsSlots edges x 2 float4 (this lane's slices of
  // the neighbour's 256-float chunk), filled by cp.async two 4-edge groups
  // ahead; shared address of slot t, vector q: my_ring + (t * 2 + q) * 512
  const uint32_t my_ring =
      smem_u32(dots_ring) + static_cast<uint32_t>((group * kDotsSlots * 2 * 32 + lane) * 16);
  int64_t row;
  int e0, e1;
  bool seg;
  if (static_cast<int>(blockIdx.x) < seg_blocks) {
    const int64_t sidx = static_cast<int64_t>(blockIdx.x) * (kThreads / 32) + group;
    if (sidx >= n_seg) return;
    row = seg_row[sidx];
    e0 = seg_begin[sidx];
    e1 = seg_end[sidx];
    seg = true;
  } else {  // light rows in the plan's length order
    const int64_t li = static_cast<int64_t>(blockIdx.x - seg_blocks) * (kThreads / 32) + group;
    if (li >= n_light) return;
    row = light[li];
    e0 = rowptr[row];
    e1 = rowptr[row + 1];
    seg = false;
  }
  const int k = e0 + lane;
  const bool valid = k < e1;
  const int cnt = e1 - e0;
  const int c = valid ? __ldg(col + k) : 0;
  const int64_t HD = static_cast<int64_t>(H) * D;
  for (int h0 = 0; h0 < H; h0 += kAggHB) {
    float mine[kAggHB];
#pragma unroll
    for (int hh = 0; hh < kAggHB; ++hh) mine[hh] = 0.0f;
    for (int64_t f0 = 0; f0 < D; f0 += kChunk) {
      float4 u[kAggHB][2];
#pragma unroll
      for (int hh = 0; hh < kAggHB; ++hh)
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const int64_t fi = f0 + static_cast<int64_t>(lane + q * 32) * 4;
          u[hh][q] = (h0 + hh < H && fi < D)
                         ? ld_vec<4>(U + row * HD + static_cast<int64_t>(h0 + hh) * D + fi)
                         : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      // slices past D get no copies: zero this lane's slots for them once
      // per chunk, so that every edge's slices are read without a select (a
      // ring slot of an edge past the item's end keeps stale values, but its
      // dots are reduced separately from every other edge's and never used)
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int64_t fi = f0 + static_cast<int64_t>(lane + q * 32) * 4;
        if (fi >= D) {
#pragma unroll
          for (int t = 0; t < kDotsSlots; ++t)
            dots_ring[(group * kDotsSlots * 2 + t * 2 + q) * 32 + lane] =
                make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      // 4 edges per pass (their neighbour chunks copied two passes ahead),
      // and the 16 (edge, head) partial dots are reduced across the warp by a
      // transposed butterfly (each level halves the values a lane carries),
      // leaving the total of value m = 4*edge + head on lanes 2m and 2m+1.
      auto issue = [&](int t0i) {  // copies of the 4-edge group starting at t0i
#pragma unroll
        for (int e4 = 0; e4 < 4; ++e4) {
          const int t = t0i + e4;
          const int ct = __shfl_sync(kFullMask, c, t < 32 ? t : 31);
          if (t >= cnt) continue;
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const int64_t fi = f0 + static_cast<int64_t>(lane + q * 32) * 4;
            if (fi < D)
              cp_async16_s(my_ring + static_cast<uint32_t>(((t % kDotsSlots) * 2 + q) * 512),
                           X + static_cast<int64_t>(ct) * D + fi);
          }
        }
        cp_async_commit();
      };
      issue(0);
      issue(4);
      for (int t0 = 0; t0 < cnt; t0 += 4) {
        cp_async_wait<1>();  // this group's copies have landed (the next may be in flight)
        float v[16];
#pragma unroll
        for (int e4 = 0; e4 < 4; ++e4) {  // one edge's slices in registers at a time
          const int t = t0 + e4;
          float4 x[2];
#pragma unroll
          for (int q = 0; q < 2; ++q)
            x[q] = lds_f4(my_ring + static_cast<uint32_t>(((t % kDotsSlots) * 2 + q) * 512));
#pragma unroll
          for (int hh = 0; hh < kAggHB; ++hh) {
            float d = 0.0f;
#pragma unroll
            for (int q = 0; q < 2; ++q) {
              d = fmaf(u[hh][q].x, x[q].x, d);
              d = fmaf(u[hh][q].y, x[q].y, d);
              d = fmaf(u[hh][q].z, x[q].z, d);
              d = fmaf(u[hh][q].w, x[q].w, d);
            }
            v[e4 * 4 + hh] = d;
          }
        }
        issue(t0 + 8);  // into the slots just read
#pragma unroll
        for (int level = 0; level < 4; ++level) {
          const int half = 8 >> level;                 // values kept after this level
          const int off = 16 >> level;                 // lane distance
          const bool upper = (lane & off) != 0;
#pragma unroll
          for (int j = 0; j < half; ++j) {
            const float keep = upper ? v[j + half] : v[j];
            const float send = upper ? v[j] : v[j + half];
            v[j] = keep + __shfl_xor_sync(kFullMask, send, off);
          }
        }
        const float tot = v[0] + __shfl_xor_sync(kFullMask, v[0], 1);
        // lane t0 + e4 (the edge's owner) collects its 4 heads
        const int e_mine = lane - t0;
        const bool owner = e_mine >= 0 && e_mine < 4;
#pragma unroll
        for (int hh = 0; hh < kAggHB; ++hh) {
          const int src = 2 * ((owner ? e_mine : 0) * 4 + hh);
          const float d = __shfl_sync(kFullMask, tot, src);
          if (owner) mine[hh] += d;
        }
      }
      cp_async_wait<0>();  // the ring is reused by the next chunk
    }
#pragma unroll
    for (int hh = 0; hh < kAggHB; ++hh) {
      const int h = h0 + hh;
      if (h >= H) break;
      const int64_t o = static_cast<int64_t>(k) * H + h;
      if (seg) {
        if (valid) glog[o] = mine[hh];
        continue;
      }
      const float ad = attn_row[row * H + h];
      const float m = emax[row * H + h], s = esum[row * H + h];
      EdgeSoft es{0.0f, 0.0f, false};
      if (valid)
        es = edge_soft(ad, __ldg(attn_col + static_cast<int64_t>(c) * H + h), m, s, slope, p, seed,
                       static_cast<uint64_t>(k) * H + h, mine[hh]);
      const float wsum = group_sum<32>(valid ? es.soft * es.ge : 0.0f, kFullMask);
      float gout = 0.0f;
      if (valid) {
        gout = es.soft * (es.ge - wsum);
        if (es.neg) gout *= slope;
        glog[o] = gout;
      }
      const float grow = group_sum<32>(gout, kFullMask);
      if (lane == 0) grad_attn_row[row * H + h] = grow;
    }
  }
}

// The edge weights [nnz, H] (CSR edge order) of every row item of the plan.
template <bool STATS>
int launch_edge_weights(const cign_gat_plan* pl, int H, const float* attn_row,
                        const float* attn_col, float* emax, float* esum, float slope, float p,
                        Seed seed, float* wts, cudaStream_t s) {
  const SegList& rs = pl->rows;
  const int64_t seg_blocks = (rs.n_seg + kThreads / 32 - 1) / (kThreads / 32);
  const int64_t grid = seg_blocks + (rs.n_light + kThreads / 32 - 1) / (kThreads / 32);
  CIGN_REQUIRE(grid < (1ll << 31), CIGN_ERR_UNSUPPORTED, "gat edge weights: grid too large");
  gat_edge_weights_kernel<STATS><<<static_cast<unsigned>(grid), kThreads, 0, s>>>(
      static_cast<int>(rs.n_light), rs.light_row(), H, pl->rowptr, pl->col, rs.seg_row(), rs.seg_begin(),
      rs.seg_end(), static_cast<int>(rs.n_seg), static_cast<int>(seg_blocks), attn_row, attn_col,
      emax, esum, slope, p, seed, wts);
  CIGN_CHECK_LAUNCH("gat_edge_weights_kernel");
  return CIGN_OK;
}

template <int VPL, int MODE>
int launch_agg(const cign_gat_plan* pl, const SegList& sl, int H, int64_t D, const int* ptr,
               const int* idx, const int* perm, const float* wts, const float* src,
               float* out, float* partial, const float* glog, float* gcol, float* pcol,
               cudaStream_t s) {
  using Cfg = AggCfg<VPL>;
  const int64_t seg_blocks = (sl.n_seg + Cfg::kGroups - 1) / Cfg::kGroups;
  const int64_t grid = seg_blocks + (sl.n_light + Cfg::kGroups - 1) / Cfg::kGroups;
  const int64_t tiles = (D + Cfg::kTile - 1) / Cfg::kTile;
  CIGN_REQUIRE(grid < (1ll << 31) && tiles < 65536, CIGN_ERR_UNSUPPORTED, "gat_agg: grid too large");
  static_assert(Cfg::kSmem <= 48 * 1024, "aggregation ring exceeds the default shared memory");
  const dim3 g(static_cast<unsigned>(grid), static_cast<unsigned>(tiles));
  if (H <= kAggHB)
    gat_agg_kernel<VPL, MODE, true><<<g, kThreads, Cfg::kSmem, s>>>(
        static_cast<int>(sl.n_light), sl.light_row(), H, D, ptr, idx, perm, sl.seg_row(), sl.seg_begin(),
        sl.seg_end(), static_cast<int>(sl.n_seg), static_cast<int>(seg_blocks), wts, src, out,
        partial, glog, gcol, pcol);
  else
    gat_agg_kernel<VPL, MODE, false><<<g, kThreads, Cfg::kSmem, s>>>(
        static_cast<int>(sl.n_light), sl.light_row(), H, D, ptr, idx, perm, sl.seg_row(), sl.seg_begin(),
        sl.seg_end(), static_cast<int>(sl.n_seg), static_cast<int>(seg_blocks), wts, src, out,
        partial, glog, gcol, pcol);
  CIGN_CHECK_LAUNCH("gat_agg_kernel");
  return launch_seg_combine(sl, H, D, partial, MODE == 1 ? pcol : nullptr, out,
                            MODE == 1 ? gcol : nullptr, s);
}

// aggregate-first workspace: hub partials [max(n_seg rows, n_seg cols), H*D]
// | column-hub logit partials [n_seg cols, H] | grad_logit [nnz, H]
struct AggLayout {
  size_t partial, pcol, glog, wts, total;
};
AggLayout agg_layout(const cign_gat_plan* pl, int H, int64_t D, int64_t C) {
  AggLayout L;
  // the aggregation kernels' own (kAggSegLen-edge) items: their hub partials
  const size_t part = std::max(static_cast<size_t>(pl->agg_rows.n_seg) * D,
                               static_cast<size_t>(pl->agg_cols.n_seg) * C);
  L.partial = 0;
  L.pcol = rnd(part * H * sizeof(float));
  L.glog = L.pcol + rnd(static_cast<size_t>(pl->agg_cols.n_seg) * H * sizeof(float));
  L.wts = L.glog + rnd(static_cast<size_t>(pl->nnz) * H * sizeof(float));
  L.total = L.wts + rnd(static_cast<size_t>(pl->nnz) * H * sizeof(float)) + 256;
  return L;
}

int check_agg(const cign_gat_plan* pl, int H, int64_t D, std::initializer_list<const void*> ptrs,
              const char* name) {
  int rc = check_plan(pl, H, D, name);
  if (rc) return rc;
  CIGN_REQUIRE(D % 4 == 0, CIGN_ERR_UNSUPPORTED, "%s: D must be a multiple of 4", name);
  for (const void* q : ptrs) {
    CIGN_REQUIRE(q != nullptr, CIGN_ERR_NULL_POINTER, "%s: NULL tensor argument", name);
    CIGN_REQUIRE(aligned16(q), CIGN_ERR_ALIGNMENT, "%s: tensors must be 16-byte aligned", name);
  }
  return CIGN_OK;
}

}  // namespace
}  // namespace cign

using namespace cign;

extern "C" {

int cign_gat_plan_create(int64_t n, int64_t nnz, const int32_t* rowptr, const int32_t* col,
                         const int32_t* colptr, const int32_t* row, const int32_t* perm,
                         cign_gat_plan** out) {
  return cign_gat_plan_create_rect(n, n, nnz, rowptr, col, colptr, row, perm, out);
}

int cign_gat_plan_create_rect(int64_t n, int64_t n_cols, int64_t nnz, const int32_t* rowptr,
                              const int32_t* col, const int32_t* colptr, const int32_t* row,
                              const int32_t* perm, cign_gat_plan** out) {
  CIGN_REQUIRE(out != nullptr, CIGN_ERR_NULL_POINTER, "gat_plan_create: out is NULL");
  *out = nullptr;
  CIGN_REQUIRE(n >= 0 && n_cols >= 0 && nnz >= 0 && n < (1ll << 31) && n_cols < (1ll << 31) &&
                   nnz < (1ll << 31),
               CIGN_ERR_INVALID_ARGUMENT, "gat_plan_create: bad sizes");
  CIGN_REQUIRE(rowptr != nullptr && colptr != nullptr, CIGN_ERR_NULL_POINTER,
               "gat_plan_create: rowptr/colptr is NULL");
  CIGN_REQUIRE(nnz == 0 || (col && row && perm), CIGN_ERR_NULL_POINTER,
               "gat_plan_create: col/row/perm is NULL");
  int* bad_d = nullptr;
  CIGN_CHECK_CUDA(cudaMalloc(&bad_d, sizeof(int)), "gat_plan_create: cudaMalloc");
  cudaMemset(bad_d, 0, sizeof(int));
  const int64_t work = std::max<int64_t>(std::max<int64_t>(std::max(n, n_cols), nnz), 1);
  const int blocks = static_cast<int>(std::min<int64_t>((work + 255) / 256, 4096));
  gat_validate_kernel<<<blocks, 256>>>(n, n_cols, nnz, rowptr, col, colptr, row, perm, bad_d);
  cudaError_t le = cudaGetLastError();
  int bad = 0;
  cudaError_t ce = cudaMemcpy(&bad, bad_d, sizeof(int), cudaMemcpyDeviceToHost);
  cudaFree(bad_d);
  if (le != cudaSuccess || ce != cudaSuccess)
    return set_error(CIGN_ERR_CUDA, "gat_plan_create: validation failed: %s",
                     cudaGetErrorString(le != cudaSuccess ? le : ce));
  CIGN_REQUIRE(bad == 0, CIGN_ERR_INVALID_ARGUMENT,
               "gat_plan_create: malformed graph (code 0x%x: 1/2 pointer arrays not monotone, "
               "4/8 index out of range, 16/32/64 perm inconsistent with CSR/CSC, 128/256 "
               "pointer ends)", bad);
  cign_gat_plan* pl = new cign_gat_plan();
  pl->n = n;
  pl->n_cols = n_cols;
  pl->nnz = nnz;
  pl->rowptr = rowptr;
  pl->col = col;
  pl->colptr = colptr;
  pl->row = row;
  pl->perm = perm;
  cudaGetDevice(&pl->device);
  int rc = build_segments(rowptr, n, kSegLen, &pl->rows);
  if (rc == CIGN_OK) rc = build_segments(colptr, n_cols, kSegLen, &pl->cols);
  if (rc == CIGN_OK) rc = build_segments(rowptr, n, kAggSegLen, &pl->agg_rows);
  if (rc == CIGN_OK) rc = build_segments(colptr, n_cols, kAggSegLen, &pl->agg_cols);
  if (rc != CIGN_OK) {
    free_segments(&pl->rows);
    free_segments(&pl->cols);
    free_segments(&pl->agg_rows);
    free_segments(&pl->agg_cols);
    delete pl;
    return rc;
  }
  *out = pl;
  clear_error();
  return CIGN_OK;
}

int cign_gat_plan_destroy(cign_gat_plan* pl) {
  if (pl == nullptr) return CIGN_OK;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(pl->device);
  free_segments(&pl->rows);
  free_segments(&pl->cols);
  free_segments(&pl->agg_rows);
  free_segments(&pl->agg_cols);
  cudaSetDevice(prev);
  delete pl;
  return CIGN_OK;
}

int cign_gat_plan_get_info(const cign_gat_plan* pl, int64_t* info) {
  CIGN_REQUIRE(pl != nullptr && info != nullptr, CIGN_ERR_NULL_POINTER,
               "gat_plan_get_info: NULL argument");
  info[0] = pl->n;
  info[1] = pl->nnz;
  info[2] = pl->rows.n_heavy;
  info[3] = pl->cols.n_heavy;
  info[4] = pl->rows.max_len;
  info[5] = pl->cols.max_len;
  info[6] = pl->rows.n_seg;
  info[7] = pl->cols.n_seg;
  return CIGN_OK;
}

size_t cign_gat_fwd_workspace_bytes(const cign_gat_plan* pl, int32_t heads, int32_t channels) {
  if (pl == nullptr || channels <= 0) return 0;
  return fwd_ws_bytes(pl, channels);
}

int cign_gat_fwd(const cign_gat_plan* pl, int32_t heads, int32_t channels, const float* attn_row,
                 const float* attn_col, const float* in_feat, const float* bias,
                 float negative_slope, float attn_drop, uint64_t seed_value, const uint64_t* seed_ptr,
                 float* out, float* pre,
                 float* edge_max, float* edge_sum, void* ws, size_t ws_bytes,
                 cign_stream_t stream) {
  const Seed seed{seed_value, seed_ptr};
  int rc = check_plan(pl, heads, channels, "gat_fwd");
  if (rc) return rc;
  CIGN_REQUIRE(pl->n == pl->n_cols, CIGN_ERR_UNSUPPORTED,
               "gat_fwd: needs a square graph (rectangular plans: cign_gat_agg_*)");
  CIGN_REQUIRE(attn_drop >= 0.0f && attn_drop < 1.0f, CIGN_ERR_INVALID_ARGUMENT,
               "gat_fwd: attn_drop must be in [0,1)");
  if (pl->n == 0) return CIGN_OK;
  CIGN_REQUIRE(attn_row && attn_col && in_feat && bias && out && pre && edge_max && edge_sum,
               CIGN_ERR_NULL_POINTER, "gat_fwd: NULL tensor argument");
  const size_t need = fwd_ws_bytes(pl, channels);
  CIGN_REQUIRE(ws_bytes >= need && (need == 0 || ws != nullptr), CIGN_ERR_INVALID_ARGUMENT,
               "gat_fwd: workspace too small (%zu < %zu bytes)", ws_bytes, need);
  const int64_t C = channels;
  float* partial = static_cast<float*>(ws);
  const bool v4 = C % 4 == 0 && aligned16(in_feat) && aligned16(out) && aligned16(pre) &&
                  aligned16(bias) && aligned16(partial);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool tma_ok = v4 && heads <= kRingMaxH && C <= 1024 &&
                      static_cast<uint64_t>(heads) * C * 4 <= kTmaSlotMax;
  if (tma_ok) {
    int* ctl = reinterpret_cast<int*>(static_cast<char*>(ws) + need - 256);
    CIGN_TMA_VPL_DISPATCH(C / 4, return (launch_fwd_tma_vpl<P_>(pl, heads, C, attn_row, attn_col, in_feat, bias, negative_slope, attn_drop, seed, out, pre, edge_max, edge_sum, partial, ctl, s)));
  }
  if (v4 && heads <= kRingMaxH) {
    int* counter = reinterpret_cast<int*>(static_cast<char*>(ws) + need - 256);
    return launch_fwd_ring(pl, heads, C, attn_row, attn_col, in_feat, bias, negative_slope,
                           attn_drop, seed, out, pre, edge_max, edge_sum, partial, counter, s);
  }
  if (v4) {
    CIGN_GAT_DISPATCH(4, C / 4, return (launch_fwd_cfg<V_, P_, L_>(pl, heads, C, attn_row, attn_col, in_feat, bias, negative_slope, attn_drop, seed, out, pre, edge_max, edge_sum, partial, s)));
  }
  CIGN_GAT_DISPATCH(1, C, return (launch_fwd_cfg<V_, P_, L_>(pl, heads, C, attn_row, attn_col, in_feat, bias, negative_slope, attn_drop, seed, out, pre, edge_max, edge_sum, partial, s)));
  return CIGN_OK;
}

size_t cign_gat_bwd_workspace_bytes(const cign_gat_plan* pl, int32_t heads, int32_t channels) {
  if (pl == nullptr || heads <= 0 || channels <= 0) return 0;
  return bwd_layout(pl, heads, channels).total;
}

int cign_gat_bwd(const cign_gat_plan* pl, int32_t heads, int32_t channels, const float* attn_row,
                 const float* attn_col, const float* in_feat, const float* pre,
                 const float* edge_max, const float* edge_sum, const float* grad_y,
                 float negative_slope, float attn_drop, uint64_t seed_value, const uint64_t* seed_ptr,
                 float* grad_feat,
                 float* grad_attn_row, float* grad_attn_col, float* grad_bias, void* ws,
                 size_t ws_bytes, cign_stream_t stream) {
  const Seed seed{seed_value, seed_ptr};
  int rc = check_plan(pl, heads, channels, "gat_bwd");
  if (rc) return rc;
  CIGN_REQUIRE(pl->n == pl->n_cols, CIGN_ERR_UNSUPPORTED,
               "gat_bwd: needs a square graph (rectangular plans: cign_gat_agg_*)");
  CIGN_REQUIRE(attn_drop >= 0.0f && attn_drop < 1.0f, CIGN_ERR_INVALID_ARGUMENT,
               "gat_bwd: attn_drop must be in [0,1)");
  const int64_t C = channels;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (pl->n == 0) return CIGN_OK;
  CIGN_REQUIRE(attn_row && attn_col && in_feat && pre && edge_max && edge_sum && grad_y &&
                   grad_feat && grad_attn_row && grad_attn_col && grad_bias,
               CIGN_ERR_NULL_POINTER, "gat_bwd: NULL tensor argument");
  const BwdLayout L = bwd_layout(pl, heads, C);
  CIGN_REQUIRE(ws != nullptr && ws_bytes >= L.total, CIGN_ERR_INVALID_ARGUMENT,
               "gat_bwd: workspace too small (%zu < %zu bytes)", ws_bytes, L.total);
  CIGN_REQUIRE(aligned16(ws), CIGN_ERR_ALIGNMENT, "gat_bwd: ws must be 16-byte aligned");
  char* w = static_cast<char*>(ws);
  float* gpre = reinterpret_cast<float*>(w + L.gpre);
  float* glog = reinterpret_cast<float*>(w + L.glog);
  float* csum = reinterpret_cast<float*>(w + L.csum);
  float* pfeat = reinterpret_cast<float*>(w + L.pfeat);
  float* pcol = reinterpret_cast<float*>(w + L.pcol);
  int* counters = reinterpret_cast<int*>(w + L.counters);
  const bool v4 = C % 4 == 0 && aligned16(in_feat) && aligned16(pre) && aligned16(grad_y) &&
                  aligned16(grad_feat);
  const bool tma_ok = v4 && heads <= kRingMaxH && C <= 1024 &&
                      static_cast<uint64_t>(heads) * C * 4 <= kTmaSlotMax;
  if (tma_ok) {
    CIGN_TMA_VPL_DISPATCH(C / 4, rc = (launch_bwd_rows_tma_vpl<P_>(pl, heads, C, attn_row, attn_col, in_feat, pre, edge_max, edge_sum, grad_y, negative_slope, attn_drop, seed, gpre, glog, grad_attn_row, counters, s)));
    if (rc) return rc;
    CIGN_TMA_VPL_DISPATCH(C / 4, rc = (launch_bwd_cols_tma_vpl<P_>(pl, heads, C, attn_row, attn_col, edge_max, edge_sum, gpre, glog, negative_slope, attn_drop, seed, grad_feat, grad_attn_col, pfeat, pcol, counters + 2, s)));
    if (rc) return rc;
    return colsum_f32(gpre, pl->n, C, csum, grad_bias, s);
  }
  if (v4 && heads <= kRingMaxH) {
    rc = launch_bwd_rows_ring(pl, heads, C, attn_row, attn_col, in_feat, pre, edge_max, edge_sum,
                              grad_y, negative_slope, attn_drop, seed, gpre, glog, grad_attn_row,
                              counters, s);
    if (rc) return rc;
    rc = launch_bwd_cols_ring(pl, heads, C, attn_row, attn_col, edge_max, edge_sum, gpre, glog,
                              negative_slope, attn_drop, seed, grad_feat, grad_attn_col, pfeat,
                              pcol, counters + 1, s);
    if (rc) return rc;
    return colsum_f32(gpre, pl->n, C, csum, grad_bias, s);
  }
  if (v4) {
    CIGN_GAT_DISPATCH(4, C / 4, rc = (launch_bwd_rows_cfg<V_, P_, L_>(pl, heads, C, attn_row, attn_col, in_feat, pre, edge_max, edge_sum, grad_y, negative_slope, attn_drop, seed, gpre, glog, grad_attn_row, s)));
  } else {
    CIGN_GAT_DISPATCH(1, C, rc = (launch_bwd_rows_cfg<V_, P_, L_>(pl, heads, C, attn_row, attn_col, in_feat, pre, edge_max, edge_sum, grad_y, negative_slope, attn_drop, seed, gpre, glog, grad_attn_row, s)));
  }
  if (rc) return rc;
  // Heads per K2 pass: keep HB * VPL <= 16 accumulator vectors.
  if (v4) {
    const int64_t fv = C / 4;
    if (fv > 128) {
      CIGN_GAT_DISPATCH(4, fv, rc = (launch_bwd_cols_cfg<V_, P_, L_, 2>(pl, heads, C, attn_row, attn_col, edge_max, edge_sum, gpre, glog, negative_slope, attn_drop, seed, grad_feat, grad_attn_col, pfeat, pcol, s)));
    } else {
      CIGN_GAT_DISPATCH(4, fv, rc = (launch_bwd_cols_cfg<V_, P_, L_, 4>(pl, heads, C, attn_row, attn_col, edge_max, edge_sum, gpre, glog, negative_slope, attn_drop, seed, grad_feat, grad_attn_col, pfeat, pcol, s)));
    }
  } else {
    CIGN_GAT_DISPATCH(1, C, rc = (launch_bwd_cols_cfg<V_, P_, L_, 2>(pl, heads, C, attn_row, attn_col, edge_max, edge_sum, gpre, glog, negative_slope, attn_drop, seed, grad_feat, grad_attn_col, pfeat, pcol, s)));
  }
  if (rc) return rc;
  return colsum_f32(gpre, pl->n, C, csum, grad_bias, s);
}

int cign_gat_dropout_mask(int64_t nnz, int32_t heads, float attn_drop, uint64_t seed_value, const uint64_t* seed_ptr,
                          uint8_t* mask, cign_stream_t stream) {
  const Seed seed{seed_value, seed_ptr};
  CIGN_REQUIRE(nnz >= 0 && heads >= 1, CIGN_ERR_INVALID_ARGUMENT, "gat_dropout_mask: bad sizes");
  const int64_t total = nnz * heads;
  if (total == 0) return CIGN_OK;
  CIGN_REQUIRE(mask != nullptr, CIGN_ERR_NULL_POINTER, "gat_dropout_mask: mask is NULL");
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 65535));
  gat_mask_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(total, attn_drop, seed,
                                                                         mask);
  CIGN_CHECK_LAUNCH("gat_mask_kernel");
  return CIGN_OK;
}

size_t cign_gat_agg_workspace_bytes(const cign_gat_plan* pl, int32_t heads, int64_t dim,
                                    int64_t channels) {
  if (pl == nullptr || heads <= 0 || dim <= 0 || channels <= 0) return 0;
  return agg_layout(pl, heads, dim, channels).total;
}

// Body of cign_gat_agg_fwd / cign_gat_agg_fwd_w: the edge weights go to
// wts_out when it is given (kept by the caller for the backward), else to
// the workspace.
static int gat_agg_fwd_impl(const cign_gat_plan* pl, int32_t heads, int64_t dim,
                            const float* attn_row, const float* attn_col, const float* x,
                            float negative_slope, float attn_drop, uint64_t seed_value,
                            const uint64_t* seed_ptr, float* z, float* edge_max, float* edge_sum,
                            float* wts_out, void* ws, size_t ws_bytes, cign_stream_t stream) {
  const Seed seed{seed_value, seed_ptr};
  int rc = check_agg(pl, heads, dim, {x, z, ws}, "gat_agg_fwd");
  if (rc) return rc;
  CIGN_REQUIRE(attn_drop >= 0.0f && attn_drop < 1.0f, CIGN_ERR_INVALID_ARGUMENT,
               "gat_agg_fwd: attn_drop must be in [0,1)");
  CIGN_REQUIRE(attn_row && attn_col && edge_max && edge_sum, CIGN_ERR_NULL_POINTER,
               "gat_agg_fwd: NULL tensor argument");
  const AggLayout L = agg_layout(pl, heads, dim, dim);
  CIGN_REQUIRE(ws_bytes >= L.total, CIGN_ERR_INVALID_ARGUMENT,
               "gat_agg_fwd: workspace too small (%zu < %zu bytes)", ws_bytes, L.total);
  if (pl->n == 0) return CIGN_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* partial = reinterpret_cast<float*>(static_cast<char*>(ws) + L.partial);
  float* wts = wts_out != nullptr ? wts_out
                                  : reinterpret_cast<float*>(static_cast<char*>(ws) + L.wts);
  rc = launch_hub_stats(pl, heads, attn_row, attn_col, negative_slope, edge_max, edge_sum, s);
  if (rc) return rc;
  rc = launch_edge_weights<true>(pl, heads, attn_row, attn_col, edge_max, edge_sum,
                                 negative_slope, attn_drop, seed, wts, s);
  if (rc) return rc;
  if (dim <= 128)
    return launch_agg<1, 0>(pl, pl->agg_rows, heads, dim, pl->rowptr, pl->col, nullptr, wts, x, z,
                            partial, nullptr, nullptr, nullptr, s);
  return launch_agg<2, 0>(pl, pl->agg_rows, heads, dim, pl->rowptr, pl->col, nullptr, wts, x, z,
                          partial, nullptr, nullptr, nullptr, s);
}

int cign_gat_agg_fwd(const cign_gat_plan* pl, int32_t heads, int64_t dim, const float* attn_row,
                     const float* attn_col, const float* x, float negative_slope, float attn_drop,
                     uint64_t seed_value, const uint64_t* seed_ptr,
                     float* z, float* edge_max, float* edge_sum, void* ws,
                     size_t ws_bytes, cign_stream_t stream) {
  return gat_agg_fwd_impl(pl, heads, dim, attn_row, attn_col, x, negative_slope, attn_drop,
                          seed_value, seed_ptr, z, edge_max, edge_sum, nullptr, ws, ws_bytes,
                          stream);
}

int cign_gat_agg_fwd_w(const cign_gat_plan* pl, int32_t heads, int64_t dim,
                       const float* attn_row, const float* attn_col, const float* x,
                       float negative_slope, float attn_drop, uint64_t seed_value,
                       const uint64_t* seed_ptr, float* z, float* edge_max, float* edge_sum,
                       float* wts, void* ws, size_t ws_bytes, cign_stream_t stream) {
  CIGN_REQUIRE(wts != nullptr || pl == nullptr || pl->nnz == 0, CIGN_ERR_NULL_POINTER,
               "gat_agg_fwd_w: NULL edge-weight buffer");
  return gat_agg_fwd_impl(pl, heads, dim, attn_row, attn_col, x, negative_slope, attn_drop,
                          seed_value, seed_ptr, z, edge_max, edge_sum, wts, ws, ws_bytes, stream);
}

int cign_gat_agg_fwd_bf16(const cign_gat_plan* pl, int32_t heads, int64_t dim,
                          const float* attn_row, const float* attn_col, const void* x,
                          float negative_slope, float attn_drop, uint64_t seed_value,
                          const uint64_t* seed_ptr, float* z, float* edge_max, float* edge_sum,
                          void* ws, size_t ws_bytes, cign_stream_t stream) {
  const Seed seed{seed_value, seed_ptr};
  int rc = check_agg(pl, heads, dim, {x, z, ws}, "gat_agg_fwd_bf16");
  if (rc) return rc;
  CIGN_REQUIRE(dim % 8 == 0, CIGN_ERR_UNSUPPORTED, "gat_agg_fwd_bf16: D must be a multiple of 8");
  CIGN_REQUIRE(attn_drop >= 0.0f && attn_drop < 1.0f, CIGN_ERR_INVALID_ARGUMENT,
               "gat_agg_fwd_bf16: attn_drop must be in [0,1)");
  CIGN_REQUIRE(attn_row && attn_col && edge_max && edge_sum, CIGN_ERR_NULL_POINTER,
               "gat_agg_fwd_bf16: NULL tensor argument");
  const AggLayout L = agg_layout(pl, heads, dim, dim);
  CIGN_REQUIRE(ws_bytes >= L.total, CIGN_ERR_INVALID_ARGUMENT,
               "gat_agg_fwd_bf16: workspace too small (%zu < %zu bytes)", ws_bytes, L.total);
  if (pl->n == 0) return CIGN_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* partial = reinterpret_cast<float*>(static_cast<char*>(ws) + L.partial);
  rc = launch_hub_stats(pl, heads, attn_row, attn_col, negative_slope, edge_max, edge_sum, s);
  if (rc) return rc;
  const SegList& sl = pl->agg_rows;  // the fp32 aggregation's items: same sums
  const int64_t seg_blocks = (sl.n_seg + kThreads / 32 - 1) / (kThreads / 32);
  const int64_t grid = seg_blocks + (sl.n_light + kThreads / 32 - 1) / (kThreads / 32);
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  // 256-feature tiles (512 bytes of bf16 per edge): the 4-head fp32
  // accumulator of a 512-feature tile would need ~120 registers
  constexpr int VPL = 1;
  const size_t smem = static_cast<size_t>(kThreads / 32) * kAggStages * VPL * 32 * 16;
  const dim3 g(static_cast<unsigned>(grid), static_cast<unsigned>((dim + 255) / 256));
  gat_agg_fwd_bf16_kernel<VPL><<<g, kThreads, smem, s>>>(
      static_cast<int>(sl.n_light), sl.light_row(), heads, dim, pl->rowptr, pl->col, sl.seg_row(),
      sl.seg_begin(), sl.seg_end(), static_cast<int>(sl.n_seg), static_cast<int>(seg_blocks),
      attn_row, attn_col,
      edge_max, edge_sum, xb, negative_slope, attn_drop, seed, z, partial);
  CIGN_CHECK_LAUNCH("gat_agg_fwd_bf16_kernel");
  return launch_seg_combine(sl, heads, dim, partial, nullptr, z, nullptr, s);
}

// Body of cign_gat_agg_bwd / cign_gat_agg_bwd_w: with wts_in (the forward's
// edge weights) K2 reads them instead of forming them again.
static int gat_agg_bwd_impl(const cign_gat_plan* pl, int32_t heads, int64_t dim,
                            int64_t channels, const float* attn_row, const float* attn_col,
                            const float* x, const float* edge_max, const float* edge_sum,
                            const float* grad_z, const float* grad_pre, float negative_slope,
                            float attn_drop, uint64_t seed_value, const uint64_t* seed_ptr,
                            const float* wts_in, float* grad_feat, float* grad_attn_row,
                            float* grad_attn_col, void* ws, size_t ws_bytes,
                            cign_stream_t stream) {
  const Seed seed{seed_value, seed_ptr};
  int rc = check_agg(pl, heads, dim, {x, grad_z, ws}, "gat_agg_bwd");
  if (rc) return rc;
  rc = check_agg(pl, heads, channels, {grad_pre, grad_feat}, "gat_agg_bwd");
  if (rc) return rc;
  CIGN_REQUIRE(attn_drop >= 0.0f && attn_drop < 1.0f, CIGN_ERR_INVALID_ARGUMENT,
               "gat_agg_bwd: attn_drop must be in [0,1)");
  CIGN_REQUIRE(attn_row && attn_col && edge_max && edge_sum && grad_attn_row && grad_attn_col,
               CIGN_ERR_NULL_POINTER, "gat_agg_bwd: NULL tensor argument");
  const AggLayout L = agg_layout(pl, heads, dim, channels);
  CIGN_REQUIRE(ws_bytes >= L.total, CIGN_ERR_INVALID_ARGUMENT,
               "gat_agg_bwd: workspace too small (%zu < %zu bytes)", ws_bytes, L.total);
  if (pl->n == 0) return CIGN_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* w = static_cast<char*>(ws);
  float* partial = reinterpret_cast<float*>(w + L.partial);
  float* pcol = reinterpret_cast<float*>(w + L.pcol);
  float* glog = reinterpret_cast<float*>(w + L.glog);
  // K1: dots U[i,h,:].X[j,:] and the softmax backward (rows)
  const SegList& rs = pl->rows;
  const int64_t seg_blocks = (rs.n_seg + kThreads / 32 - 1) / (kThreads / 32);
  const int64_t grid = seg_blocks + (rs.n_light + kThreads / 32 - 1) / (kThreads / 32);
  CIGN_REQUIRE(grid < (1ll << 31), CIGN_ERR_UNSUPPORTED, "gat_agg_bwd: grid too large");
  {  // 64 KB of dynamic shared memory: opt in once per device
    static std::mutex mu;
    static bool set[64] = {false};
    int dev = 0;
    CIGN_CHECK_CUDA(cudaGetDevice(&dev), "gat_agg_bwd: cudaGetDevice");
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 0 || dev >= 64 || !set[dev]) {
      CIGN_CHECK_CUDA(cudaFuncSetAttribute(gat_agg_dots_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(kDotsSmem)),
                      "gat_agg_bwd: shared-memory opt-in");
      if (dev >= 0 && dev < 64) set[dev] = true;
    }
  }
  gat_agg_dots_kernel<<<static_cast<unsigned>(grid), kThreads, kDotsSmem, s>>>(
      static_cast<int>(rs.n_light), rs.light_row(), heads, dim, pl->rowptr, pl->col, rs.seg_row(), rs.seg_begin(),
      rs.seg_end(), static_cast<int>(rs.n_seg), static_cast<int>(seg_blocks), attn_row, attn_col,
      edge_max, edge_sum, grad_z, x, negative_slope, attn_drop, seed, glog, grad_attn_row);
  CIGN_CHECK_LAUNCH("gat_agg_dots_kernel");
  rc = launch_bwd_hub_rows(pl, heads, channels, attn_row, attn_col, nullptr, edge_max, edge_sum,
                           nullptr, negative_slope, attn_drop, seed, nullptr, glog, grad_attn_row,
                           s);
  if (rc) return rc;
  // K2: grad_feat[j,h,:] = sum_i w g_pre[i,:] / H and grad_attn_col (columns),
  // with the forward's edge weights or ones formed again from its statistics
  const float* wts = wts_in;
  if (wts == nullptr) {
    float* wk = reinterpret_cast<float*>(w + L.wts);
    rc = launch_edge_weights<false>(pl, heads, attn_row, attn_col, const_cast<float*>(edge_max),
                                    const_cast<float*>(edge_sum), negative_slope, attn_drop, seed,
                                    wk, s);
    if (rc) return rc;
    wts = wk;
  }
  if (channels <= 128)
    return launch_agg<1, 1>(pl, pl->agg_cols, heads, channels, pl->colptr, pl->row, pl->perm, wts,
                            grad_pre, grad_feat, partial, glog, grad_attn_col, pcol, s);
  return launch_agg<2, 1>(pl, pl->agg_cols, heads, channels, pl->colptr, pl->row, pl->perm, wts,
                          grad_pre, grad_feat, partial, glog, grad_attn_col, pcol, s);
}

int cign_gat_agg_bwd(const cign_gat_plan* pl, int32_t heads, int64_t dim, int64_t channels,
                     const float* attn_row, const float* attn_col, const float* x,
                     const float* edge_max, const float* edge_sum, const float* grad_z,
                     const float* grad_pre, float negative_slope, float attn_drop,
                     uint64_t seed_value, const uint64_t* seed_ptr, float* grad_feat,
                     float* grad_attn_row, float* grad_attn_col, void* ws, size_t ws_bytes,
                     cign_stream_t stream) {
  return gat_agg_bwd_impl(pl, heads, dim, channels, attn_row, attn_col, x, edge_max, edge_sum,
                          grad_z, grad_pre, negative_slope, attn_drop, seed_value, seed_ptr,
                          nullptr, grad_feat, grad_attn_row, grad_attn_col, ws, ws_bytes, stream);
}

int cign_gat_agg_bwd_w(const cign_gat_plan* pl, int32_t heads, int64_t dim, int64_t channels,
                       const float* attn_row, const float* attn_col, const float* x,
                       const float* edge_max, const float* edge_sum, const float* grad_z,
                       const float* grad_pre, const float* wts, float negative_slope,
                       float attn_drop, uint64_t seed_value, const uint64_t* seed_ptr,
                       float* grad_feat, float* grad_attn_row, float* grad_attn_col, void* ws,
                       size_t ws_bytes, cign_stream_t stream) {
  CIGN_REQUIRE(wts != nullptr || pl == nullptr || pl->nnz == 0, CIGN_ERR_NULL_POINTER,
               "gat_agg_bwd_w: NULL edge-weight buffer");
  return gat_agg_bwd_impl(pl, heads, dim, channels, attn_row, attn_col, x, edge_max, edge_sum,
                          grad_z, grad_pre, negative_slope, attn_drop, seed_value, seed_ptr, wts,
                          grad_feat, grad_attn_row, grad_attn_col, ws, ws_bytes, stream);
}

}  // extern "C"
