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
#include <algorithm>

#include "common.cuh"

struct cign_gat_plan {
  int64_t n;
  int64_t nnz;
  const int32_t* rowptr;
  const int32_t* col;
  const int32_t* colptr;
  const int32_t* row;
  const int32_t* perm;
  cign::SegList rows;  // hub destination rows (CSR)
  cign::SegList cols;  // hub source columns (CSC)
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
__device__ __forceinline__ float block_sum(float v, float* scratch) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) scratch[w] = v;
  __syncthreads();
  float r = 0.0f;
#pragma unroll
  for (int i = 0; i < kThreads / 32; ++i) r += scratch[i];
  return r;
}
__device__ __forceinline__ float block_max(float v, float* scratch) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) scratch[w] = v;
  __syncthreads();
  float r = scratch[0];
#pragma unroll
  for (int i = 1; i < kThreads / 32; ++i) r = fmaxf(r, scratch[i]);
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
// Hub rows: one CTA per row computes the per-head max / exp-sum.
__global__ void __launch_bounds__(kThreads)
gat_hub_stats_kernel(int H, const int* __restrict__ rowptr, const int* __restrict__ col,
                     const int* __restrict__ hub_row, const float* __restrict__ attn_row,
                     const float* __restrict__ attn_col, float slope,
                     float* __restrict__ emax, float* __restrict__ esum) {
  __shared__ float scratch[32];
  const int64_t row = hub_row[blockIdx.x];
  const int e0 = rowptr[row], e1 = rowptr[row + 1];
  for (int h = 0; h < H; ++h) {
    const float ad = attn_row[row * H + h];
    float m = kNegInit;
    for (int e = e0 + threadIdx.x; e < e1; e += kThreads)
      m = fmaxf(m, leaky_f(ad + attn_col[static_cast<int64_t>(col[e]) * H + h], slope));
    m = block_max(m, scratch);
    float s = 0.0f;
    for (int e = e0 + threadIdx.x; e < e1; e += kThreads)
      s += expf(leaky_f(ad + attn_col[static_cast<int64_t>(col[e]) * H + h], slope) - m);
    s = block_sum(s, scratch);
    if (threadIdx.x == 0) {
      emax[row * H + h] = m;
      esum[row * H + h] = s;
    }
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
               const float* __restrict__ bias, float slope, float p, uint64_t seed,
               float* __restrict__ out, float* __restrict__ pre, float* __restrict__ emax,
               float* __restrict__ esum, float* __restrict__ partial) {
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

// One CTA per hub row: acc = sum of segment partials (segment order),
// pre = acc / H + bias, out = SiLU(pre).
__global__ void __launch_bounds__(kThreads)
gat_fwd_combine_kernel(int H, int64_t C, const int* __restrict__ hub_row,
                       const int* __restrict__ hub_first, const float* __restrict__ partial,
                       const float* __restrict__ bias, float* __restrict__ pre,
                       float* __restrict__ out) {
  const int64_t row = hub_row[blockIdx.x];
  const int s0 = hub_first[blockIdx.x], s1 = hub_first[blockIdx.x + 1];
  const float hf = static_cast<float>(H);
  for (int64_t c = threadIdx.x; c < C; c += kThreads) {
    float a = 0.0f;
    for (int s = s0; s < s1; ++s) a += partial[static_cast<int64_t>(s) * C + c];
    const float pj = a / hf + bias[c];
    pre[row * C + c] = pj;
    out[row * C + c] = silu_f(pj);
  }
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
                    float slope, float p, uint64_t seed, float* __restrict__ gpre,
                    float* __restrict__ glog, float* __restrict__ grad_attn_row) {
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

// One CTA per hub row: write its g_pre row and run the softmax backward over
// its edges (dots already in glog from the segment groups).
__global__ void __launch_bounds__(kThreads)
gat_bwd_hub_rows_kernel(int H, int64_t C, const int* __restrict__ rowptr,
                        const int* __restrict__ col, const int* __restrict__ hub_row,
                        const float* __restrict__ attn_row, const float* __restrict__ attn_col,
                        const float* __restrict__ pre, const float* __restrict__ emax,
                        const float* __restrict__ esum, const float* __restrict__ grad_y,
                        float slope, float p, uint64_t seed, float* __restrict__ gpre,
                        float* __restrict__ glog, float* __restrict__ grad_attn_row) {
  __shared__ float scratch[32];
  const int64_t row = hub_row[blockIdx.x];
  for (int64_t c = threadIdx.x; c < C; c += kThreads)
    gpre[row * C + c] = grad_y[row * C + c] * silu_grad_f(pre[row * C + c]);
  const int e0 = rowptr[row], e1 = rowptr[row + 1];
  for (int h = 0; h < H; ++h) {
    const float ad = attn_row[row * H + h];
    const float m = emax[row * H + h], s = esum[row * H + h];
    float wsum = 0.0f;
    for (int e = e0 + threadIdx.x; e < e1; e += kThreads) {
      const EdgeSoft es = edge_soft(ad, attn_col[static_cast<int64_t>(col[e]) * H + h], m, s, slope,
                                    p, seed, static_cast<uint64_t>(e) * H + h,
                                    glog[static_cast<int64_t>(e) * H + h]);
      wsum += es.soft * es.ge;
    }
    wsum = block_sum(wsum, scratch);
    float grow = 0.0f;
    for (int e = e0 + threadIdx.x; e < e1; e += kThreads) {
      const int64_t o = static_cast<int64_t>(e) * H + h;
      const EdgeSoft es = edge_soft(ad, attn_col[static_cast<int64_t>(col[e]) * H + h], m, s, slope,
                                    p, seed, static_cast<uint64_t>(e) * H + h, glog[o]);
      float gout = es.soft * (es.ge - wsum);
      if (es.neg) gout *= slope;
      glog[o] = gout;
      grow += gout;
    }
    grow = block_sum(grow, scratch);
    if (threadIdx.x == 0) grad_attn_row[row * H + h] = grow;
  }
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
                    float slope, float p, uint64_t seed, float* __restrict__ grad_feat,
                    float* __restrict__ grad_attn_col, float* __restrict__ pfeat,
                    float* __restrict__ pcol) {
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

// One CTA per hub column: sum the segment partials in segment order.
__global__ void __launch_bounds__(kThreads)
gat_bwd_cols_combine_kernel(int H, int64_t C, const int* __restrict__ hub_col,
                            const int* __restrict__ hub_first, const float* __restrict__ pfeat,
                            const float* __restrict__ pcol, float* __restrict__ grad_feat,
                            float* __restrict__ grad_attn_col) {
  const int64_t j = hub_col[blockIdx.x];
  const int s0 = hub_first[blockIdx.x], s1 = hub_first[blockIdx.x + 1];
  const int64_t HC = static_cast<int64_t>(H) * C;
  for (int64_t k = threadIdx.x; k < HC; k += kThreads) {
    float a = 0.0f;
    for (int s = s0; s < s1; ++s) a += pfeat[static_cast<int64_t>(s) * HC + k];
    grad_feat[j * HC + k] = a;
  }
  for (int h = threadIdx.x; h < H; h += kThreads) {
    float a = 0.0f;
    for (int s = s0; s < s1; ++s) a += pcol[static_cast<int64_t>(s) * H + h];
    grad_attn_col[j * H + h] = a;
  }
}

// ------------------------------------------------------------ misc kernels
__global__ void gat_mask_kernel(int64_t total, float p, uint64_t seed,
                                uint8_t* __restrict__ mask) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += stride)
    mask[i] = gat_keep(seed, static_cast<uint64_t>(i), p) ? 1 : 0;
}

__global__ void gat_validate_kernel(int64_t n, int64_t nnz, const int* __restrict__ rowptr,
                                    const int* __restrict__ col, const int* __restrict__ colptr,
                                    const int* __restrict__ row, const int* __restrict__ perm,
                                    int* __restrict__ bad) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  for (int64_t i = t0; i < n; i += stride) {
    if (rowptr[i] > rowptr[i + 1]) atomicOr(bad, 1);
    if (colptr[i] > colptr[i + 1]) atomicOr(bad, 2);
  }
  for (int64_t e = t0; e < nnz; e += stride) {
    const int c = col[e];
    if (c < 0 || c >= n) atomicOr(bad, 4);
    const int r = row[e];
    if (r < 0 || r >= n) { atomicOr(bad, 8); continue; }
    const int pe = perm[e];
    if (pe < 0 || pe >= nnz) { atomicOr(bad, 16); continue; }
    // The CSR edge perm[e] must lie in row r's CSR range.
    if (pe < rowptr[r] || pe >= rowptr[r + 1]) atomicOr(bad, 32);
  }
  // CSC position pos of column j must map to a CSR edge whose column is j.
  for (int64_t j = t0; j < n; j += stride) {
    const int lo = max(colptr[j], 0);
    const int hi = min(static_cast<int64_t>(colptr[j + 1]), nnz);
    for (int pos = lo; pos < hi; ++pos) {
      const int pe = perm[pos];
      if (pe >= 0 && pe < nnz && col[pe] != j) { atomicOr(bad, 64); break; }
    }
  }
  if (t0 == 0) {
    if (rowptr[0] != 0 || rowptr[n] != nnz) atomicOr(bad, 128);
    if (colptr[0] != 0 || colptr[n] != nnz) atomicOr(bad, 256);
  }
}

// ------------------------------------------------------------ dispatch
size_t rnd(size_t b) { return (b + 255) / 256 * 256; }

template <int VEC, int VPL, int LPR>
int launch_fwd_cfg(const cign_gat_plan* pl, int H, int64_t C, const float* attn_row,
                   const float* attn_col, const float* x, const float* bias, float slope, float p,
                   uint64_t seed, float* out, float* pre, float* emax, float* esum, float* partial,
                   cudaStream_t s) {
  using Cfg = GatCfg<VEC, VPL, LPR>;
  const SegList& sl = pl->rows;
  if (sl.n_heavy > 0) {
    gat_hub_stats_kernel<<<static_cast<unsigned>(sl.n_heavy), kThreads, 0, s>>>(
        H, pl->rowptr, pl->col, sl.heavy_row(), attn_row, attn_col, slope, emax, esum);
    CIGN_CHECK_LAUNCH("gat_hub_stats_kernel");
  }
  const int64_t seg_blocks = (sl.n_seg + Cfg::kGroups - 1) / Cfg::kGroups;
  const int64_t grid = seg_blocks + (pl->n + Cfg::kGroups - 1) / Cfg::kGroups;
  const size_t smem = static_cast<size_t>(Cfg::kGroups) * 2 * H * sizeof(float);
  gat_fwd_kernel<VEC, VPL, LPR><<<static_cast<unsigned>(grid), kThreads, smem, s>>>(
      static_cast<int>(pl->n), H, C, pl->rowptr, pl->col, sl.seg_row(), sl.seg_begin(),
      sl.seg_end(), static_cast<int>(sl.n_seg), static_cast<int>(seg_blocks), attn_row, attn_col,
      x, bias, slope, p, seed, out, pre, emax, esum, partial);
  CIGN_CHECK_LAUNCH("gat_fwd_kernel");
  if (sl.n_heavy > 0) {
    gat_fwd_combine_kernel<<<static_cast<unsigned>(sl.n_heavy), kThreads, 0, s>>>(
        H, C, sl.heavy_row(), sl.heavy_first(), partial, bias, pre, out);
    CIGN_CHECK_LAUNCH("gat_fwd_combine_kernel");
  }
  return CIGN_OK;
}

template <int VEC, int VPL, int LPR>
int launch_bwd_rows_cfg(const cign_gat_plan* pl, int H, int64_t C, const float* attn_row,
                        const float* attn_col, const float* x, const float* pre,
                        const float* emax, const float* esum, const float* gy, float slope,
                        float p, uint64_t seed, float* gpre, float* glog, float* grow,
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
  if (sl.n_heavy > 0) {
    gat_bwd_hub_rows_kernel<<<static_cast<unsigned>(sl.n_heavy), kThreads, 0, s>>>(
        H, C, pl->rowptr, pl->col, sl.heavy_row(), attn_row, attn_col, pre, emax, esum, gy, slope,
        p, seed, gpre, glog, grow);
    CIGN_CHECK_LAUNCH("gat_bwd_hub_rows_kernel");
  }
  return CIGN_OK;
}

template <int VEC, int VPL, int LPR, int HB>
int launch_bwd_cols_cfg(const cign_gat_plan* pl, int H, int64_t C, const float* attn_row,
                        const float* attn_col, const float* emax, const float* esum,
                        const float* gpre, const float* glog, float slope, float p, uint64_t seed,
                        float* gfeat, float* gcol, float* pfeat, float* pcol, cudaStream_t s) {
  using Cfg = GatCfg<VEC, VPL, LPR>;
  const SegList& sl = pl->cols;
  const int64_t seg_blocks = (sl.n_seg + Cfg::kGroups - 1) / Cfg::kGroups;
  const int64_t grid = seg_blocks + (pl->n + Cfg::kGroups - 1) / Cfg::kGroups;
  gat_bwd_cols_kernel<VEC, VPL, LPR, HB><<<static_cast<unsigned>(grid), kThreads, 0, s>>>(
      static_cast<int>(pl->n), H, C, pl->colptr, pl->row, pl->perm, sl.seg_row(), sl.seg_begin(),
      sl.seg_end(), static_cast<int>(sl.n_seg), static_cast<int>(seg_blocks), attn_row, attn_col,
      emax, esum, gpre, glog, slope, p, seed, gfeat, gcol, pfeat, pcol);
  CIGN_CHECK_LAUNCH("gat_bwd_cols_kernel");
  if (sl.n_heavy > 0) {
    gat_bwd_cols_combine_kernel<<<static_cast<unsigned>(sl.n_heavy), kThreads, 0, s>>>(
        H, C, sl.heavy_row(), sl.heavy_first(), pfeat, pcol, gfeat, gcol);
    CIGN_CHECK_LAUNCH("gat_bwd_cols_combine_kernel");
  }
  return CIGN_OK;
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

size_t fwd_ws_bytes(const cign_gat_plan* pl, int64_t C) {
  return rnd(static_cast<size_t>(pl->rows.n_seg) * C * sizeof(float));
}

// backward workspace: g_pre [N*C] | grad_logit [nnz*H] | colsum partials |
// column-segment partials [n_seg*(H*C)] | [n_seg*H]
struct BwdLayout {
  size_t gpre, glog, csum, pfeat, pcol, total;
};
BwdLayout bwd_layout(const cign_gat_plan* pl, int H, int64_t C) {
  BwdLayout L;
  L.gpre = 0;
  L.glog = L.gpre + rnd(static_cast<size_t>(pl->n) * C * sizeof(float));
  L.csum = L.glog + rnd(static_cast<size_t>(pl->nnz) * H * sizeof(float));
  L.pfeat = L.csum + rnd(static_cast<size_t>(colsum_chunks(pl->n)) * C * sizeof(float));
  L.pcol = L.pfeat + rnd(static_cast<size_t>(pl->cols.n_seg) * H * C * sizeof(float));
  L.total = L.pcol + rnd(static_cast<size_t>(pl->cols.n_seg) * H * sizeof(float));
  return L;
}

}  // namespace
}  // namespace cign

using namespace cign;

extern "C" {

int cign_gat_plan_create(int64_t n, int64_t nnz, const int32_t* rowptr, const int32_t* col,
                         const int32_t* colptr, const int32_t* row, const int32_t* perm,
                         cign_gat_plan** out) {
  CIGN_REQUIRE(out != nullptr, CIGN_ERR_NULL_POINTER, "gat_plan_create: out is NULL");
  *out = nullptr;
  CIGN_REQUIRE(n >= 0 && nnz >= 0 && n < (1ll << 31) && nnz < (1ll << 31),
               CIGN_ERR_INVALID_ARGUMENT, "gat_plan_create: bad sizes");
  CIGN_REQUIRE(rowptr != nullptr && colptr != nullptr, CIGN_ERR_NULL_POINTER,
               "gat_plan_create: rowptr/colptr is NULL");
  CIGN_REQUIRE(nnz == 0 || (col && row && perm), CIGN_ERR_NULL_POINTER,
               "gat_plan_create: col/row/perm is NULL");
  int* bad_d = nullptr;
  CIGN_CHECK_CUDA(cudaMalloc(&bad_d, sizeof(int)), "gat_plan_create: cudaMalloc");
  cudaMemset(bad_d, 0, sizeof(int));
  const int64_t work = std::max<int64_t>(std::max<int64_t>(n, nnz), 1);
  const int blocks = static_cast<int>(std::min<int64_t>((work + 255) / 256, 4096));
  gat_validate_kernel<<<blocks, 256>>>(n, nnz, rowptr, col, colptr, row, perm, bad_d);
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
  pl->nnz = nnz;
  pl->rowptr = rowptr;
  pl->col = col;
  pl->colptr = colptr;
  pl->row = row;
  pl->perm = perm;
  cudaGetDevice(&pl->device);
  int rc = build_segments(rowptr, n, kSegLen, &pl->rows);
  if (rc == CIGN_OK) rc = build_segments(colptr, n, kSegLen, &pl->cols);
  if (rc != CIGN_OK) {
    free_segments(&pl->rows);
    free_segments(&pl->cols);
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
                 float negative_slope, float attn_drop, uint64_t seed, float* out, float* pre,
                 float* edge_max, float* edge_sum, void* ws, size_t ws_bytes,
                 cign_stream_t stream) {
  int rc = check_plan(pl, heads, channels, "gat_fwd");
  if (rc) return rc;
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
                 float negative_slope, float attn_drop, uint64_t seed, float* grad_feat,
                 float* grad_attn_row, float* grad_attn_col, float* grad_bias, void* ws,
                 size_t ws_bytes, cign_stream_t stream) {
  int rc = check_plan(pl, heads, channels, "gat_bwd");
  if (rc) return rc;
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
  const bool v4 = C % 4 == 0 && aligned16(in_feat) && aligned16(pre) && aligned16(grad_y) &&
                  aligned16(grad_feat);
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

int cign_gat_dropout_mask(int64_t nnz, int32_t heads, float attn_drop, uint64_t seed,
                          uint8_t* mask, cign_stream_t stream) {
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

}  // extern "C"
