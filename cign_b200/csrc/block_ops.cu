// Block side ops for any hidden width D: dropout + LayerNorm, add +
// LayerNorm, dropout + gamma-scaled residual, forward and backward.
//
// Reference: fused_block_ops.py (generic kernels, 1 <= D <= 256, inline
// CUDA :15) and fused_block_ops_ext/fused_block_ops_cuda.cu (D = 256).
// Semantics kept: dropout keep iff (splitmix64(seed ^ idx*0xD2B74407B1CE6E93)
// >> 11) * 2^-53 >= p with idx = n*D + d and kept values scaled by 1/(1-p);
// LayerNorm with biased variance, y = (q - mean) * rsqrt(var + eps) * w + b.
//
// A group of LPR lanes owns one row and holds it in registers (D <= the
// group's register tile), so mean and variance are two in-register passes.
// The dropout mask is recomputed from (seed, idx) in backward, never stored.
// Parameter gradients (LN weight/bias, gamma) are accumulated per lane in
// registers over a fixed chunk of rows, reduced across the CTA's groups in
// shared memory in a fixed order, then summed over chunks by a second tiny
// kernel: deterministic, no atomics.
#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace cign {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxGroups = 32;  // kThreads / smallest LPR (8)

template <int VEC, int VPL, int LPR>
struct RowCfg {
  static constexpr int kGroups = kThreads / LPR;
  static constexpr int kTile = LPR * VPL * VEC;
};

template <int LPR>
__device__ __forceinline__ unsigned row_group_mask() {
  return LPR == 32 ? kFullMask
                   : (((1u << LPR) - 1u) << ((threadIdx.x & 31) / LPR * LPR));
}
template <int LPR>
__device__ __forceinline__ float gsum(float v, unsigned gmask) {
#pragma unroll
  for (int o = LPR / 2; o > 0; o >>= 1) v += __shfl_xor_sync(gmask, v, o, LPR);
  return v;
}

// Row chunks of the parameter-gradient reductions (one CTA each): at most
// this many -- three per SM, the residency of the 80-register backward
// kernels, so that all chunks run in one wave (a second, partial wave left
// most SMs idle) -- each a multiple of 8 rows.
constexpr int64_t kLnChunkTarget = 444;
// silu_add_ln_bwd_kernel keeps three parameter partials and its row in
// registers (~128): two CTAs per SM, so its chunks target two per SM.
constexpr int64_t kSiluLnChunkTarget = 296;
int64_t rows_per_chunk(int64_t n, int64_t target = kLnChunkTarget) {
  int64_t r = (n + target - 1) / target;
  r = std::max<int64_t>(r, 8);
  return (r + 7) / 8 * 8;
}
int64_t num_chunks(int64_t n, int64_t target = kLnChunkTarget) {
  return (n + rows_per_chunk(n, target) - 1) / rows_per_chunk(n, target);
}

// ---------------------------------------------------------------- forward
// MODE 0: dropout-LN (x, seed, p);  MODE 1: add-LN (a + b).
template <int MODE, int VEC, int VPL, int LPR>
__global__ void __launch_bounds__(kThreads)
ln_fwd_kernel(int64_t n, int64_t D, const float* __restrict__ x, const float* __restrict__ x2,
              const float* __restrict__ w, const float* __restrict__ b, float p, float eps,
              Seed seed_in, float* __restrict__ y, float* __restrict__ mean,
              float* __restrict__ rstd) {
  const uint64_t seed = seed_in;
  using V = typename VecT<VEC>::type;
  using Cfg = RowCfg<VEC, VPL, LPR>;
  const int lig = threadIdx.x % LPR;
  const unsigned gmask = row_group_mask<LPR>();
  const int64_t row = static_cast<int64_t>(blockIdx.x) * Cfg::kGroups + threadIdx.x / LPR;
  if (row >= n) return;
  const float scale = p > 0.0f ? 1.0f / (1.0f - p) : 1.0f;
  V q[VPL];
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    const int64_t d = static_cast<int64_t>(lig + k * LPR) * VEC;
    vzero(q[k]);
    if (d < D) {
      const V xv = ld_vec<VEC>(x + row * D + d);
      if (MODE == 0) {
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          const bool keep = block_keep(seed, static_cast<uint64_t>(row * D + d + j), p);
          vel(q[k], j) = keep ? vel(xv, j) * scale : 0.0f;
        }
      } else {
        const V x2v = ld_vec<VEC>(x2 + row * D + d);
#pragma unroll
        for (int j = 0; j < VEC; ++j) vel(q[k], j) = vel(xv, j) + vel(x2v, j);
      }
#pragma unroll
      for (int j = 0; j < VEC; ++j) s += vel(q[k], j);
    }
  }
  const float mu = gsum<LPR>(s, gmask) / static_cast<float>(D);
  float v = 0.0f;
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    const int64_t d = static_cast<int64_t>(lig + k * LPR) * VEC;
    if (d < D) {
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        const float cdev = vel(q[k], j) - mu;
        v += cdev * cdev;
      }
    }
  }
  const float rs = rsqrtf(gsum<LPR>(v, gmask) / static_cast<float>(D) + eps);
  if (lig == 0) {
    mean[row] = mu;
    rstd[row] = rs;
  }
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    const int64_t d = static_cast<int64_t>(lig + k * LPR) * VEC;
    if (d < D) {
      const V wv = ldg_vec<VEC>(w + d);
      const V bv = ldg_vec<VEC>(b + d);
      V o;
#pragma unroll
      for (int j = 0; j < VEC; ++j) vel(o, j) = (vel(q[k], j) - mu) * rs * vel(wv, j) + vel(bv, j);
      st_vec(y + row * D + d, o);
    }
  }
}

// ---------------------------------------------------------------- backward
// grad wrt the normalised input (dq) plus per-chunk partials of
// sum(gy * xhat) and sum(gy) for the LN weight and bias.  With addend !=
// NULL the row's addend [n, D] is added to the written gradient (a second
// consumer's gradient of the same input, e.g. a residual branch).
template <int MODE, int VEC, int VPL, int LPR>
__global__ void __launch_bounds__(kThreads, VPL <= 4 ? 3 : 1)
ln_bwd_kernel(int64_t n, int64_t D, int64_t rpc, const float* __restrict__ gy,
              const float* __restrict__ x, const float* __restrict__ x2,
              const float* __restrict__ w, const float* __restrict__ mean,
              const float* __restrict__ rstd, float p, Seed seed_in,
              const float* __restrict__ addend, float* __restrict__ gx,
              float* __restrict__ pw, float* __restrict__ pb) {
  const uint64_t seed = seed_in;
  using V = typename VecT<VEC>::type;
  using Cfg = RowCfg<VEC, VPL, LPR>;
  __shared__ float red[kThreads * VPL * VEC];  // per thread: VPL*VEC partials
  const int lig = threadIdx.x % LPR;
  const int group = threadIdx.x / LPR;
  const unsigned gmask = row_group_mask<LPR>();
  const float scale = p > 0.0f ? 1.0f / (1.0f - p) : 1.0f;
  const float Df = static_cast<float>(D);
  V aw[VPL], ab[VPL];
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    vzero(aw[k]);
    vzero(ab[k]);
  }
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rpc;
  const int64_t r1 = (r0 + rpc < n) ? (r0 + rpc) : n;
  static_assert(VPL * VEC <= 32, "one keep bit per element of a lane's row slice");
  // Two passes over each row: the first forms the row sums and the parameter
  // partials, the second re-reads x (and x2), gy (this warp's own recent
  // loads: L1 hits) and writes grad x, so a lane keeps no row arrays (only
  // the dropout keep bits, hashed once per element).
  for (int64_t row = r0 + group; row < r1; row += Cfg::kGroups) {
    const float mu = mean[row], rs = rstd[row];
    uint32_t keep_bits = 0;  // MODE 0: the dropout keep bits
    float s1 = 0.0f, s2 = 0.0f;
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int64_t d = static_cast<int64_t>(lig + k * LPR) * VEC;
      if (d < D) {
        const V xv = ld_vec<VEC>(x + row * D + d);
        const V gv = ld_vec<VEC>(gy + row * D + d);
        const V wv = ldg_vec<VEC>(w + d);
        V x2v;
        if (MODE == 1) x2v = ld_vec<VEC>(x2 + row * D + d);
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          float qv;
          if (MODE == 0) {
            const bool keep = block_keep(seed, static_cast<uint64_t>(row * D + d + j), p);
            keep_bits |= static_cast<uint32_t>(keep) << (k * VEC + j);
            qv = keep ? vel(xv, j) * scale : 0.0f;
          } else {
            qv = vel(xv, j) + vel(x2v, j);
          }
          const float xhat = (qv - mu) * rs;
          const float dnorm = vel(gv, j) * vel(wv, j);
          s1 += dnorm;
          s2 += dnorm * xhat;
          vel(aw[k], j) += vel(gv, j) * xhat;
          vel(ab[k], j) += vel(gv, j);
        }
      }
    }
    s1 = gsum<LPR>(s1, gmask);
    s2 = gsum<LPR>(s2, gmask);
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int64_t d = static_cast<int64_t>(lig + k * LPR) * VEC;
      if (d < D) {
        const V xv = ld_vec<VEC>(x + row * D + d);
        const V gv = ld_vec<VEC>(gy + row * D + d);
        const V wv = ldg_vec<VEC>(w + d);
        V x2v;
        if (MODE == 1) x2v = ld_vec<VEC>(x2 + row * D + d);
        V o;
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          const bool keep = MODE == 0 ? ((keep_bits >> (k * VEC + j)) & 1u) != 0 : true;
          const float qv = MODE == 0 ? (keep ? vel(xv, j) * scale : 0.0f) : vel(xv, j) + vel(x2v, j);
          const float xhat = (qv - mu) * rs;
          const float dnorm = vel(gv, j) * vel(wv, j);
          const float dq = (rs / Df) * (Df * dnorm - s1 - xhat * s2);
          vel(o, j) = MODE == 0 ? (keep ? dq * scale : 0.0f) : dq;
        }
        if (addend != nullptr) vadd(o, ld_vec<VEC>(addend + row * D + d));
        st_vec(gx + row * D + d, o);
      }
    }
  }
  // Reduce the groups' column partials in a fixed order.
  for (int pass = 0; pass < 2; ++pass) {
    V(&acc)[VPL] = pass == 0 ? aw : ab;
    float* out = pass == 0 ? pw : pb;
    __syncthreads();
#pragma unroll
    for (int k = 0; k < VPL; ++k)
#pragma unroll
      for (int j = 0; j < VEC; ++j) red[(group * Cfg::kTile) + (lig + k * LPR) * VEC + j] = vel(acc[k], j);
    __syncthreads();
    for (int64_t d = threadIdx.x; d < D && d < Cfg::kTile; d += kThreads) {
      float t = 0.0f;
      for (int g = 0; g < Cfg::kGroups; ++g) t += red[g * Cfg::kTile + d];
      out[static_cast<int64_t>(blockIdx.x) * D + d] = t;
    }
  }
}

// y = h + gamma * dropout(g)
template <int VEC>
__global__ void gamma_fwd_kernel(int64_t n, int64_t D, const float* __restrict__ h,
                                 const float* __restrict__ g, const float* __restrict__ gamma,
                                 float p, Seed seed_in, float* __restrict__ y) {
  const uint64_t seed = seed_in;
  using V = typename VecT<VEC>::type;
  const int64_t total = n * D / VEC;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const float scale = p > 0.0f ? 1.0f / (1.0f - p) : 1.0f;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += stride) {
    const int64_t e = i * VEC;
    const int64_t d = e % D;
    const V hv = ld_vec<VEC>(h + e);
    const V gv = ld_vec<VEC>(g + e);
    const V gm = ldg_vec<VEC>(gamma + d);
    V o;
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      const bool keep = block_keep(seed, static_cast<uint64_t>(e + j), p);
      const float gd = keep ? vel(gv, j) * scale : 0.0f;
      vel(o, j) = vel(hv, j) + vel(gm, j) * gd;
    }
    st_vec(y + e, o);
  }
}

// grad_g = gy * gamma * m;  partial[chunk, d] = sum gy * g * m  (m = keep ? scale : 0)
template <int VEC, int VPL, int LPR>
__global__ void __launch_bounds__(kThreads)
gamma_bwd_kernel(int64_t n, int64_t D, int64_t rpc, const float* __restrict__ gy,
                 const float* __restrict__ g, const float* __restrict__ gamma, float p,
                 Seed seed_in, float* __restrict__ gg, float* __restrict__ partial) {
  const uint64_t seed = seed_in;
  using V = typename VecT<VEC>::type;
  using Cfg = RowCfg<VEC, VPL, LPR>;
  __shared__ float red[kThreads * VPL * VEC];
  const int lig = threadIdx.x % LPR;
  const int group = threadIdx.x / LPR;
  const float scale = p > 0.0f ? 1.0f / (1.0f - p) : 1.0f;
  V acc[VPL];
#pragma unroll
  for (int k = 0; k < VPL; ++k) vzero(acc[k]);
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rpc;
  const int64_t r1 = (r0 + rpc < n) ? (r0 + rpc) : n;
  for (int64_t row = r0 + group; row < r1; row += Cfg::kGroups) {
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int64_t d = static_cast<int64_t>(lig + k * LPR) * VEC;
      if (d < D) {
        const V gyv = ld_vec<VEC>(gy + row * D + d);
        const V gv = ld_vec<VEC>(g + row * D + d);
        const V gm = ldg_vec<VEC>(gamma + d);
        V o;
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          const bool keep = block_keep(seed, static_cast<uint64_t>(row * D + d + j), p);
          const float m = keep ? scale : 0.0f;
          vel(o, j) = vel(gyv, j) * vel(gm, j) * m;
          vel(acc[k], j) += vel(gyv, j) * vel(gv, j) * m;
        }
        st_vec(gg + row * D + d, o);
      }
    }
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < VPL; ++k)
#pragma unroll
    for (int j = 0; j < VEC; ++j) red[(group * Cfg::kTile) + (lig + k * LPR) * VEC + j] = vel(acc[k], j);
  __syncthreads();
  for (int64_t d = threadIdx.x; d < D && d < Cfg::kTile; d += kThreads) {
    float t = 0.0f;
    for (int gi = 0; gi < Cfg::kGroups; ++gi) t += red[gi * Cfg::kTile + d];
    partial[static_cast<int64_t>(blockIdx.x) * D + d] = t;
  }
}

// ------------------------------------------------ GAT epilogue + add-LN
// The GAT layer's side ops and the block's add-LayerNorm in one pass over
// the row (model_cign.py:767-787 with the collapsed GAT's bias + SiLU,
// collapsed_gat_cuda.cu:167-173, and fused_add_layernorm):
//   pre = lin + bias;  c = SiLU(pre);  y = LayerNorm(c + h) * w + b.
// `lin` is the head-mean GAT output before its bias (the aggregate-first
// form's z @ M).  Writes pre (for the SiLU backward), y, mean and rstd; the
// SiLU output itself is never stored.  The formulas of
// cign_head_mean_bias_silu_fwd (one head) followed by cign_add_ln_fwd.
template <int VEC, int VPL, int LPR>
__global__ void __launch_bounds__(kThreads)
silu_add_ln_fwd_kernel(int64_t n, int64_t D, const float* __restrict__ lin,
                       const float* __restrict__ bias, const float* __restrict__ h,
                       const float* __restrict__ w, const float* __restrict__ b, float eps,
                       float* __restrict__ pre_out, float* __restrict__ y,
                       float* __restrict__ mean, float* __restrict__ rstd) {
  using V = typename VecT<VEC>::type;
  using Cfg = RowCfg<VEC, VPL, LPR>;
  const int lig = threadIdx.x % LPR;
  const unsigned gmask = row_group_mask<LPR>();
  const int64_t row = static_cast<int64_t>(blockIdx.x) * Cfg::kGroups + threadIdx.x / LPR;
  if (row >= n) return;
  V q[VPL];
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    const int64_t d = static_cast<int64_t>(lig + k * LPR) * VEC;
    vzero(q[k]);
    if (d < D) {
      const V lv = ld_vec<VEC>(lin + row * D + d);
      const V bv = ldg_vec<VEC>(bias + d);
      const V hv = ld_vec<VEC>(h + row * D + d);
      V pv;
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        vel(pv, j) = vel(lv, j) + vel(bv, j);
        vel(q[k], j) = silu_f(vel(pv, j)) + vel(hv, j);
        s += vel(q[k], j);
      }
      st_vec(pre_out + row * D + d, pv);
    }
  }
  const float mu = gsum<LPR>(s, gmask) / static_cast<float>(D);
  float v = 0.0f;
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    const int64_t d = static_cast<int64_t>(lig + k * LPR) * VEC;
    if (d < D) {
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        const float cdev = vel(q[k], j) - mu;
        v += cdev * cdev;
      }
    }
  }
  const float rs = rsqrtf(gsum<LPR>(v, gmask) / static_cast<float>(D) + eps);
  if (lig == 0) {
    mean[row] = mu;
    rstd[row] = rs;
  }
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    const int64_t d = static_cast<int64_t>(lig + k * LPR) * VEC;
    if (d < D) {
      const V wv = ldg_vec<VEC>(w + d);
      const V bv = ldg_vec<VEC>(b + d);
      V o;
#pragma unroll
      for (int j = 0; j < VEC; ++j) vel(o, j) = (vel(q[k], j) - mu) * rs * vel(wv, j) + vel(bv, j);
      st_vec(y + row * D + d, o);
    }
  }
}

// Backward of silu_add_ln_fwd: grad_z = dLN/d(c + h) (the gradient of h, and
// of the SiLU output c), grad_pre = grad_z * SiLU'(pre) (the gradient of lin),
// and per-chunk partials of sum(gy * xhat), sum(gy) (LN weight and bias) and
// sum(grad_pre) (the GAT bias), reduced in a fixed order like ln_bwd_kernel.
// With acc_z the row's previous grad_z is added (h's gradient from its other
// consumers).  Two passes over each row, as in ln_bwd_kernel: the first forms
// the row sums and the LN parameter partials, the second re-reads pre, h and
// gy (this warp's own recent loads) and writes grad_z and grad_pre, so a lane
// keeps only the three parameter partials (<= 128 registers: two CTAs per
// SM, the residency kSiluLnChunkTarget assumes).
template <int VEC, int VPL, int LPR>
__global__ void __launch_bounds__(kThreads, 2)
silu_add_ln_bwd_kernel(int64_t n, int64_t D, int64_t rpc, const float* __restrict__ gy,
                       const float* __restrict__ pre, const float* __restrict__ h,
                       const float* __restrict__ w, const float* __restrict__ mean,
                       const float* __restrict__ rstd, bool acc_z, float* __restrict__ gz,
                       float* __restrict__ gpre, float* __restrict__ pw,
                       float* __restrict__ pb, float* __restrict__ pbias) {
  using V = typename VecT<VEC>::type;
  using Cfg = RowCfg<VEC, VPL, LPR>;
  __shared__ float red[kThreads * VPL * VEC];
  const int lig = threadIdx.x % LPR;
  const int group = threadIdx.x / LPR;
  const unsigned gmask = row_group_mask<LPR>();
  const float Df = static_cast<float>(D);
  V aw[VPL], ab[VPL], ag[VPL];
#pragma unroll
  for (int k = 0; k < VPL; ++k) {
    vzero(aw[k]);
    vzero(ab[k]);
    vzero(ag[k]);
  }
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rpc;
  const int64_t r1 = (r0 + rpc < n) ? (r0 + rpc) : n;
  for (int64_t row = r0 + group; row < r1; row += Cfg::kGroups) {
    const float mu = mean[row], rs = rstd[row];
    float s1 = 0.0f, s2 = 0.0f;
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int64_t d = static_cast<int64_t>(lig + k * LPR) * VEC;
      if (d < D) {
        const V pv = ld_vec<VEC>(pre + row * D + d);
        const V hv = ld_vec<VEC>(h + row * D + d);
        const V gv = ld_vec<VEC>(gy + row * D + d);
        const V wv = ldg_vec<VEC>(w + d);
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          const float qv = silu_f(vel(pv, j)) + vel(hv, j);
          const float xhat = (qv - mu) * rs;
          const float dnorm = vel(gv, j) * vel(wv, j);
          s1 += dnorm;
          s2 += dnorm * xhat;
          vel(aw[k], j) += vel(gv, j) * xhat;
          vel(ab[k], j) += vel(gv, j);
        }
      }
    }
    s1 = gsum<LPR>(s1, gmask);
    s2 = gsum<LPR>(s2, gmask);
#pragma unroll
    for (int k = 0; k < VPL; ++k) {
      const int64_t d = static_cast<int64_t>(lig + k * LPR) * VEC;
      if (d < D) {
        const V pv = ld_vec<VEC>(pre + row * D + d);
        const V hv = ld_vec<VEC>(h + row * D + d);
        const V gv = ld_vec<VEC>(gy + row * D + d);
        const V wv = ldg_vec<VEC>(w + d);
        V oz, op;
        if (acc_z) oz = ld_vec<VEC>(gz + row * D + d);
        else vzero(oz);
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          // SiLU and its derivative from one sigmoid (the values silu_f and
          // silu_grad_f give, without evaluating the sigmoid twice)
          const float x = vel(pv, j);
          const float sg = sigmoid_f(x);
          const float qv = x * sg + vel(hv, j);
          const float xhat = (qv - mu) * rs;
          const float dnorm = vel(gv, j) * vel(wv, j);
          const float dq = (rs / Df) * (Df * dnorm - s1 - xhat * s2);
          vel(oz, j) += dq;
          vel(op, j) = dq * (sg * (1.0f + x * (1.0f - sg)));
          vel(ag[k], j) += vel(op, j);
        }
        st_vec(gz + row * D + d, oz);
        st_vec(gpre + row * D + d, op);
      }
    }
  }
  for (int pass = 0; pass < 3; ++pass) {
    V(&acc)[VPL] = pass == 0 ? aw : (pass == 1 ? ab : ag);
    float* out = pass == 0 ? pw : (pass == 1 ? pb : pbias);
    __syncthreads();
#pragma unroll
    for (int k = 0; k < VPL; ++k)
#pragma unroll
      for (int j = 0; j < VEC; ++j) red[(group * Cfg::kTile) + (lig + k * LPR) * VEC + j] = vel(acc[k], j);
    __syncthreads();
    for (int64_t d = threadIdx.x; d < D && d < Cfg::kTile; d += kThreads) {
      float t = 0.0f;
      for (int g = 0; g < Cfg::kGroups; ++g) t += red[g * Cfg::kTile + d];
      out[static_cast<int64_t>(blockIdx.x) * D + d] = t;
    }
  }
}

__global__ void block_mask_kernel(int64_t count, float p, Seed seed_in,
                                  uint8_t* __restrict__ mask) {
  const uint64_t seed = seed_in;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += stride)
    mask[i] = block_keep(seed, static_cast<uint64_t>(i), p) ? 1 : 0;
}

// D must fit one group's register tile: D <= 1024 with float4, <= 256 scalar.
#define CIGN_ROW_DISPATCH(VEC_, FV_, CALL)                                    \
  do {                                                                        \
    if ((FV_) <= 8) { constexpr int V_ = VEC_, P_ = 1, L_ = 8; CALL; }        \
    else if ((FV_) <= 16) { constexpr int V_ = VEC_, P_ = 1, L_ = 16; CALL; } \
    else if ((FV_) <= 32) { constexpr int V_ = VEC_, P_ = 1, L_ = 32; CALL; } \
    else if ((FV_) <= 64) { constexpr int V_ = VEC_, P_ = 2, L_ = 32; CALL; } \
    else if ((FV_) <= 128) { constexpr int V_ = VEC_, P_ = 4, L_ = 32; CALL; }\
    else { constexpr int V_ = VEC_, P_ = 8, L_ = 32; CALL; }                  \
  } while (0)

int check_rows(int64_t n, int64_t D, bool v4, const char* name) {
  CIGN_REQUIRE(n >= 0 && D >= 1, CIGN_ERR_INVALID_ARGUMENT, "%s: bad sizes", name);
  CIGN_REQUIRE(D <= (v4 ? 1024 : 256), CIGN_ERR_UNSUPPORTED,
               "%s: D=%lld exceeds the register-resident row limit (1024 for D%%4==0 with "
               "16-byte aligned tensors, else 256)", name, (long long)D);
  CIGN_REQUIRE(n < (1ll << 40), CIGN_ERR_UNSUPPORTED, "%s: too many rows", name);
  return CIGN_OK;
}

template <int MODE, int VEC, int VPL, int LPR>
int launch_ln_fwd(int64_t n, int64_t D, const float* x, const float* x2, const float* w,
                  const float* b, float p, float eps, Seed seed, float* y, float* mean,
                  float* rstd, cudaStream_t s) {
  using Cfg = RowCfg<VEC, VPL, LPR>;
  const int64_t grid = (n + Cfg::kGroups - 1) / Cfg::kGroups;
  ln_fwd_kernel<MODE, VEC, VPL, LPR><<<static_cast<unsigned>(grid), kThreads, 0, s>>>(
      n, D, x, x2, w, b, p, eps, seed, y, mean, rstd);
  CIGN_CHECK_LAUNCH("ln_fwd_kernel");
  return CIGN_OK;
}

template <int MODE, int VEC, int VPL, int LPR>
int launch_ln_bwd(int64_t n, int64_t D, const float* gy, const float* x, const float* x2,
                  const float* w, const float* mean, const float* rstd, float p, Seed seed,
                  float* gx, float* gw, float* gb, float* ws, cudaStream_t s,
                  const float* addend = nullptr) {
  const int64_t rpc = rows_per_chunk(n);
  const int64_t chunks = num_chunks(n);
  float* pw = ws;
  float* pb = ws + chunks * D;
  ln_bwd_kernel<MODE, VEC, VPL, LPR><<<static_cast<unsigned>(chunks), kThreads, 0, s>>>(
      n, D, rpc, gy, x, x2, w, mean, rstd, p, seed, addend, gx, pw, pb);
  CIGN_CHECK_LAUNCH("ln_bwd_kernel");
  return colsum_rows(pw, gw, pb, gb, chunks, D, D, s);
}

template <int VEC, int VPL, int LPR>
int launch_silu_add_ln_fwd(int64_t n, int64_t D, const float* lin, const float* bias,
                           const float* h, const float* w, const float* b, float eps, float* pre,
                           float* y, float* mean, float* rstd, cudaStream_t s) {
  using Cfg = RowCfg<VEC, VPL, LPR>;
  const int64_t grid = (n + Cfg::kGroups - 1) / Cfg::kGroups;
  silu_add_ln_fwd_kernel<VEC, VPL, LPR><<<static_cast<unsigned>(grid), kThreads, 0, s>>>(
      n, D, lin, bias, h, w, b, eps, pre, y, mean, rstd);
  CIGN_CHECK_LAUNCH("silu_add_ln_fwd_kernel");
  return CIGN_OK;
}

template <int VEC, int VPL, int LPR>
int launch_silu_add_ln_bwd(int64_t n, int64_t D, const float* gy, const float* pre,
                           const float* h, const float* w, const float* mean, const float* rstd,
                           bool acc_z, float* gz, float* gpre, float* gw, float* gb, float* gbias,
                           float* ws, cudaStream_t s) {
  const int64_t rpc = rows_per_chunk(n, kSiluLnChunkTarget);
  const int64_t chunks = num_chunks(n, kSiluLnChunkTarget);
  float* pw = ws;
  float* pb = ws + chunks * D;
  float* pbias = ws + 2 * chunks * D;
  silu_add_ln_bwd_kernel<VEC, VPL, LPR><<<static_cast<unsigned>(chunks), kThreads, 0, s>>>(
      n, D, rpc, gy, pre, h, w, mean, rstd, acc_z, gz, gpre, pw, pb, pbias);
  CIGN_CHECK_LAUNCH("silu_add_ln_bwd_kernel");
  int rc = colsum_rows(pw, gw, pb, gb, chunks, D, D, s);
  if (rc) return rc;
  return colsum_rows(pbias, gbias, nullptr, nullptr, chunks, D, D, s);
}

template <int VEC, int VPL, int LPR>
int launch_gamma_bwd(int64_t n, int64_t D, const float* gy, const float* g, const float* gamma,
                     float p, Seed seed, float* gg, float* ggamma, float* ws,
                     cudaStream_t s) {
  const int64_t rpc = rows_per_chunk(n);
  const int64_t chunks = num_chunks(n);
  gamma_bwd_kernel<VEC, VPL, LPR><<<static_cast<unsigned>(chunks), kThreads, 0, s>>>(
      n, D, rpc, gy, g, gamma, p, seed, gg, ws);
  CIGN_CHECK_LAUNCH("gamma_bwd_kernel");
  return colsum_rows(ws, ggamma, nullptr, nullptr, chunks, D, D, s);
}

}  // namespace
}  // namespace cign

using namespace cign;

extern "C" {

int cign_dropout_ln_fwd(int64_t n, int64_t d, const float* x, const float* w, const float* b,
                        float p, float eps, uint64_t seed_value, const uint64_t* seed_ptr,
                        float* y, float* mean, float* rstd,
                        cign_stream_t stream) {
  const Seed seed{seed_value, seed_ptr};
  const bool v4 = d % 4 == 0 && aligned16(x) && aligned16(w) && aligned16(b) && aligned16(y);
  int rc = check_rows(n, d, v4, "dropout_ln_fwd");
  if (rc) return rc;
  CIGN_REQUIRE(p >= 0.0f && p < 1.0f, CIGN_ERR_INVALID_ARGUMENT, "dropout_ln_fwd: p in [0,1)");
  if (n == 0) return CIGN_OK;
  CIGN_REQUIRE(x && w && b && y && mean && rstd, CIGN_ERR_NULL_POINTER, "dropout_ln_fwd: NULL");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (v4) {
    CIGN_ROW_DISPATCH(4, d / 4, return (launch_ln_fwd<0, V_, P_, L_>(n, d, x, nullptr, w, b, p, eps, seed, y, mean, rstd, s)));
  }
  CIGN_ROW_DISPATCH(1, d, return (launch_ln_fwd<0, V_, P_, L_>(n, d, x, nullptr, w, b, p, eps, seed, y, mean, rstd, s)));
  return CIGN_OK;
}

size_t cign_ln_bwd_workspace_bytes(int64_t n, int64_t d) {
  if (n <= 0) return 0;
  return static_cast<size_t>(num_chunks(n)) * d * 2 * sizeof(float);
}

int cign_dropout_ln_bwd(int64_t n, int64_t d, const float* grad_y, const float* x,
                        const float* w, const float* mean, const float* rstd, float p,
                        uint64_t seed_value, const uint64_t* seed_ptr,
                        float* grad_x, float* grad_w, float* grad_b, void* ws,
                        size_t ws_bytes, cign_stream_t stream) {
  const Seed seed{seed_value, seed_ptr};
  const bool v4 = d % 4 == 0 && aligned16(x) && aligned16(w) && aligned16(grad_y) &&
                  aligned16(grad_x);
  int rc = check_rows(n, d, v4, "dropout_ln_bwd");
  if (rc) return rc;
  CIGN_REQUIRE(grad_w && grad_b, CIGN_ERR_NULL_POINTER, "dropout_ln_bwd: NULL param grad");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n == 0) {
    CIGN_CHECK_CUDA(cudaMemsetAsync(grad_w, 0, d * sizeof(float), s), "memset");
    CIGN_CHECK_CUDA(cudaMemsetAsync(grad_b, 0, d * sizeof(float), s), "memset");
    return CIGN_OK;
  }
  CIGN_REQUIRE(grad_y && x && w && mean && rstd && grad_x, CIGN_ERR_NULL_POINTER,
               "dropout_ln_bwd: NULL");
  CIGN_REQUIRE(ws && ws_bytes >= cign_ln_bwd_workspace_bytes(n, d), CIGN_ERR_INVALID_ARGUMENT,
               "dropout_ln_bwd: workspace too small");
  float* wsf = static_cast<float*>(ws);
  if (v4) {
    CIGN_ROW_DISPATCH(4, d / 4, return (launch_ln_bwd<0, V_, P_, L_>(n, d, grad_y, x, nullptr, w, mean, rstd, p, seed, grad_x, grad_w, grad_b, wsf, s)));
  }
  CIGN_ROW_DISPATCH(1, d, return (launch_ln_bwd<0, V_, P_, L_>(n, d, grad_y, x, nullptr, w, mean, rstd, p, seed, grad_x, grad_w, grad_b, wsf, s)));
  return CIGN_OK;
}

int cign_dropout_ln_bwd_add(int64_t n, int64_t d, const float* grad_y, const float* x,
                            const float* w, const float* mean, const float* rstd, float p,
                            uint64_t seed_value, const uint64_t* seed_ptr, const float* addend,
                            float* grad_x, float* grad_w, float* grad_b, void* ws,
                            size_t ws_bytes, cign_stream_t stream) {
  const Seed seed{seed_value, seed_ptr};
  const bool v4 = d % 4 == 0 && aligned16(x) && aligned16(w) && aligned16(grad_y) &&
                  aligned16(grad_x) && aligned16(addend);
  int rc = check_rows(n, d, v4, "dropout_ln_bwd_add");
  if (rc) return rc;
  CIGN_REQUIRE(grad_w && grad_b, CIGN_ERR_NULL_POINTER, "dropout_ln_bwd_add: NULL param grad");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n == 0) {
    CIGN_CHECK_CUDA(cudaMemsetAsync(grad_w, 0, d * sizeof(float), s), "memset");
    CIGN_CHECK_CUDA(cudaMemsetAsync(grad_b, 0, d * sizeof(float), s), "memset");
    return CIGN_OK;
  }
  CIGN_REQUIRE(grad_y && x && w && mean && rstd && grad_x && addend, CIGN_ERR_NULL_POINTER,
               "dropout_ln_bwd_add: NULL");
  CIGN_REQUIRE(addend != grad_x, CIGN_ERR_INVALID_ARGUMENT,
               "dropout_ln_bwd_add: addend must not alias grad_x");
  CIGN_REQUIRE(ws && ws_bytes >= cign_ln_bwd_workspace_bytes(n, d), CIGN_ERR_INVALID_ARGUMENT,
               "dropout_ln_bwd_add: workspace too small");
  float* wsf = static_cast<float*>(ws);
  if (v4) {
    CIGN_ROW_DISPATCH(4, d / 4, return (launch_ln_bwd<0, V_, P_, L_>(n, d, grad_y, x, nullptr, w, mean, rstd, p, seed, grad_x, grad_w, grad_b, wsf, s, addend)));
  }
  CIGN_ROW_DISPATCH(1, d, return (launch_ln_bwd<0, V_, P_, L_>(n, d, grad_y, x, nullptr, w, mean, rstd, p, seed, grad_x, grad_w, grad_b, wsf, s, addend)));
  return CIGN_OK;
}

int cign_add_ln_fwd(int64_t n, int64_t d, const float* a, const float* b, const float* w,
                    const float* bias, float eps, float* y, float* mean, float* rstd,
                    cign_stream_t stream) {
  const bool v4 = d % 4 == 0 && aligned16(a) && aligned16(b) && aligned16(w) &&
                  aligned16(bias) && aligned16(y);
  int rc = check_rows(n, d, v4, "add_ln_fwd");
  if (rc) return rc;
  if (n == 0) return CIGN_OK;
  CIGN_REQUIRE(a && b && w && bias && y && mean && rstd, CIGN_ERR_NULL_POINTER, "add_ln_fwd: NULL");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (v4) {
    CIGN_ROW_DISPATCH(4, d / 4, return (launch_ln_fwd<1, V_, P_, L_>(n, d, a, b, w, bias, 0.0f, eps, 0, y, mean, rstd, s)));
  }
  CIGN_ROW_DISPATCH(1, d, return (launch_ln_fwd<1, V_, P_, L_>(n, d, a, b, w, bias, 0.0f, eps, 0, y, mean, rstd, s)));
  return CIGN_OK;
}

int cign_add_ln_bwd(int64_t n, int64_t d, const float* grad_y, const float* a, const float* b,
                    const float* w, const float* mean, const float* rstd, float* grad_z,
                    float* grad_w, float* grad_b, void* ws, size_t ws_bytes,
                    cign_stream_t stream) {
  const bool v4 = d % 4 == 0 && aligned16(a) && aligned16(b) && aligned16(w) &&
                  aligned16(grad_y) && aligned16(grad_z);
  int rc = check_rows(n, d, v4, "add_ln_bwd");
  if (rc) return rc;
  CIGN_REQUIRE(grad_w && grad_b, CIGN_ERR_NULL_POINTER, "add_ln_bwd: NULL param grad");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n == 0) {
    CIGN_CHECK_CUDA(cudaMemsetAsync(grad_w, 0, d * sizeof(float), s), "memset");
    CIGN_CHECK_CUDA(cudaMemsetAsync(grad_b, 0, d * sizeof(float), s), "memset");
    return CIGN_OK;
  }
  CIGN_REQUIRE(grad_y && a && b && w && mean && rstd && grad_z, CIGN_ERR_NULL_POINTER,
               "add_ln_bwd: NULL");
  CIGN_REQUIRE(ws && ws_bytes >= cign_ln_bwd_workspace_bytes(n, d), CIGN_ERR_INVALID_ARGUMENT,
               "add_ln_bwd: workspace too small");
  float* wsf = static_cast<float*>(ws);
  if (v4) {
    CIGN_ROW_DISPATCH(4, d / 4, return (launch_ln_bwd<1, V_, P_, L_>(n, d, grad_y, a, b, w, mean, rstd, 0.0f, 0, grad_z, grad_w, grad_b, wsf, s)));
  }
  CIGN_ROW_DISPATCH(1, d, return (launch_ln_bwd<1, V_, P_, L_>(n, d, grad_y, a, b, w, mean, rstd, 0.0f, 0, grad_z, grad_w, grad_b, wsf, s)));
  return CIGN_OK;
}

int cign_gamma_residual_fwd(int64_t n, int64_t d, const float* h, const float* g,
                            const float* gamma, float p, uint64_t seed_value, const uint64_t* seed_ptr,
                            float* y,
                            cign_stream_t stream) {
  const Seed seed{seed_value, seed_ptr};
  CIGN_REQUIRE(n >= 0 && d >= 1, CIGN_ERR_INVALID_ARGUMENT, "gamma_residual_fwd: bad sizes");
  CIGN_REQUIRE(p >= 0.0f && p < 1.0f, CIGN_ERR_INVALID_ARGUMENT, "gamma_residual_fwd: p in [0,1)");
  if (n == 0) return CIGN_OK;
  CIGN_REQUIRE(h && g && gamma && y, CIGN_ERR_NULL_POINTER, "gamma_residual_fwd: NULL");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool v4 = d % 4 == 0 && aligned16(h) && aligned16(g) && aligned16(gamma) && aligned16(y);
  const int64_t total = n * d / (v4 ? 4 : 1);
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((total + kThreads - 1) / kThreads, 148ll * 16)));
  if (v4) gamma_fwd_kernel<4><<<grid, kThreads, 0, s>>>(n, d, h, g, gamma, p, seed, y);
  else gamma_fwd_kernel<1><<<grid, kThreads, 0, s>>>(n, d, h, g, gamma, p, seed, y);
  CIGN_CHECK_LAUNCH("gamma_fwd_kernel");
  return CIGN_OK;
}

size_t cign_gamma_residual_bwd_workspace_bytes(int64_t n, int64_t d) {
  if (n <= 0) return 0;
  return static_cast<size_t>(num_chunks(n)) * d * sizeof(float);
}

int cign_gamma_residual_bwd(int64_t n, int64_t d, const float* grad_y, const float* g,
                            const float* gamma, float p, uint64_t seed_value, const uint64_t* seed_ptr,
                            float* grad_g,
                            float* grad_gamma, void* ws, size_t ws_bytes,
                            cign_stream_t stream) {
  const Seed seed{seed_value, seed_ptr};
  const bool v4 = d % 4 == 0 && aligned16(grad_y) && aligned16(g) && aligned16(gamma) &&
                  aligned16(grad_g);
  int rc = check_rows(n, d, v4, "gamma_residual_bwd");
  if (rc) return rc;
  CIGN_REQUIRE(grad_gamma != nullptr, CIGN_ERR_NULL_POINTER, "gamma_residual_bwd: NULL grad_gamma");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n == 0) {
    CIGN_CHECK_CUDA(cudaMemsetAsync(grad_gamma, 0, d * sizeof(float), s), "memset");
    return CIGN_OK;
  }
  CIGN_REQUIRE(grad_y && g && gamma && grad_g, CIGN_ERR_NULL_POINTER, "gamma_residual_bwd: NULL");
  CIGN_REQUIRE(ws && ws_bytes >= cign_gamma_residual_bwd_workspace_bytes(n, d),
               CIGN_ERR_INVALID_ARGUMENT, "gamma_residual_bwd: workspace too small");
  float* wsf = static_cast<float*>(ws);
  if (v4) {
    CIGN_ROW_DISPATCH(4, d / 4, return (launch_gamma_bwd<V_, P_, L_>(n, d, grad_y, g, gamma, p, seed, grad_g, grad_gamma, wsf, s)));
  }
  CIGN_ROW_DISPATCH(1, d, return (launch_gamma_bwd<V_, P_, L_>(n, d, grad_y, g, gamma, p, seed, grad_g, grad_gamma, wsf, s)));
  return CIGN_OK;
}

int cign_silu_add_ln_fwd(int64_t n, int64_t d, const float* lin, const float* bias,
                         const float* h, const float* w, const float* b, float eps, float* pre,
                         float* y, float* mean, float* rstd, cign_stream_t stream) {
  const bool v4 = d % 4 == 0 && aligned16(lin) && aligned16(bias) && aligned16(h) &&
                  aligned16(w) && aligned16(b) && aligned16(pre) && aligned16(y);
  int rc = check_rows(n, d, v4, "silu_add_ln_fwd");
  if (rc) return rc;
  if (n == 0) return CIGN_OK;
  CIGN_REQUIRE(lin && bias && h && w && b && pre && y && mean && rstd, CIGN_ERR_NULL_POINTER,
               "silu_add_ln_fwd: NULL");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (v4) {
    CIGN_ROW_DISPATCH(4, d / 4, return (launch_silu_add_ln_fwd<V_, P_, L_>(n, d, lin, bias, h, w, b, eps, pre, y, mean, rstd, s)));
  }
  CIGN_ROW_DISPATCH(1, d, return (launch_silu_add_ln_fwd<V_, P_, L_>(n, d, lin, bias, h, w, b, eps, pre, y, mean, rstd, s)));
  return CIGN_OK;
}

size_t cign_silu_add_ln_bwd_workspace_bytes(int64_t n, int64_t d) {
  if (n <= 0) return 0;
  return static_cast<size_t>(num_chunks(n, kSiluLnChunkTarget)) * d * 3 * sizeof(float);
}

int cign_silu_add_ln_bwd(int64_t n, int64_t d, const float* grad_y, const float* pre,
                         const float* h, const float* w, const float* mean, const float* rstd,
                         int accumulate_z, float* grad_z, float* grad_pre, float* grad_w,
                         float* grad_b, float* grad_bias, void* ws, size_t ws_bytes,
                         cign_stream_t stream) {
  const bool v4 = d % 4 == 0 && aligned16(grad_y) && aligned16(pre) && aligned16(h) &&
                  aligned16(w) && aligned16(grad_z) && aligned16(grad_pre);
  int rc = check_rows(n, d, v4, "silu_add_ln_bwd");
  if (rc) return rc;
  CIGN_REQUIRE(grad_w && grad_b && grad_bias, CIGN_ERR_NULL_POINTER,
               "silu_add_ln_bwd: NULL parameter gradient");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n == 0) {
    CIGN_CHECK_CUDA(cudaMemsetAsync(grad_w, 0, d * sizeof(float), s), "memset");
    CIGN_CHECK_CUDA(cudaMemsetAsync(grad_b, 0, d * sizeof(float), s), "memset");
    CIGN_CHECK_CUDA(cudaMemsetAsync(grad_bias, 0, d * sizeof(float), s), "memset");
    return CIGN_OK;
  }
  CIGN_REQUIRE(grad_y && pre && h && w && mean && rstd && grad_z && grad_pre,
               CIGN_ERR_NULL_POINTER, "silu_add_ln_bwd: NULL");
  CIGN_REQUIRE(ws != nullptr && ws_bytes >= cign_silu_add_ln_bwd_workspace_bytes(n, d),
               CIGN_ERR_INVALID_ARGUMENT, "silu_add_ln_bwd: workspace too small");
  float* wsf = static_cast<float*>(ws);
  if (v4) {
    CIGN_ROW_DISPATCH(4, d / 4, return (launch_silu_add_ln_bwd<V_, P_, L_>(n, d, grad_y, pre, h, w, mean, rstd, accumulate_z != 0, grad_z, grad_pre, grad_w, grad_b, grad_bias, wsf, s)));
  }
  CIGN_ROW_DISPATCH(1, d, return (launch_silu_add_ln_bwd<V_, P_, L_>(n, d, grad_y, pre, h, w, mean, rstd, accumulate_z != 0, grad_z, grad_pre, grad_w, grad_b, grad_bias, wsf, s)));
  return CIGN_OK;
}

int cign_block_dropout_mask(int64_t count, float p, uint64_t seed_value, const uint64_t* seed_ptr,
                            uint8_t* mask,
                            cign_stream_t stream) {
  const Seed seed{seed_value, seed_ptr};
  CIGN_REQUIRE(count >= 0, CIGN_ERR_INVALID_ARGUMENT, "block_dropout_mask: bad count");
  if (count == 0) return CIGN_OK;
  CIGN_REQUIRE(mask != nullptr, CIGN_ERR_NULL_POINTER, "block_dropout_mask: NULL mask");
  const int grid = static_cast<int>(std::min<int64_t>((count + 255) / 256, 65535));
  block_mask_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(count, p, seed, mask);
  CIGN_CHECK_LAUNCH("block_mask_kernel");
  return CIGN_OK;
}

}  // extern "C"

// ------------------------------------------------------------------------
// Allocation-free variant of the dropout-LayerNorm backward.
//
// Some callers cannot allocate device memory at all: for example code that
// runs as a plugin inside a host framework which owns every byte of device
// memory through its own pool and hands kernels only their input and output
// buffers, or code on a latency-critical loop where a cudaMalloc (and its
// implicit synchronisation) is not allowed.  For them the workspace of the
// parameter-gradient reduction lives in the fixed array below instead of a
// caller-provided buffer.
//
// The array holds 444 row chunks x 1024 columns x 2 partial sums (3.5 MiB);
// every GPU on which this library is loaded keeps it for the life of the
// process.  444 is the largest chunk count rows_per_chunk() can produce, so
// the limit is the hidden width: D <= 1024 (D <= 256 unless D % 4 == 0 and
// the tensors are 16-byte aligned), the same as the workspace version.
//
// The array is shared by every call in the process: two calls that overlap
// on the GPU (different streams, or different host threads) race on it and
// give undefined results; order them on one stream.  Each call overwrites
// every partial it later reads, so nothing has to be cleared between calls.
// Its device address is looked up (cudaGetSymbolAddress) on the first call
// on each device, with that device current; make that first call before any
// stream capture.  The dropout seed is a host value only (no device seed
// slot, unlike cign_dropout_ln_bwd): a captured graph that replays this call
// replays the same mask.
constexpr int64_t kStaticLnChunks = 444;
constexpr int64_t kStaticLnMaxD = 1024;
static_assert(kStaticLnChunks == kLnChunkTarget,
              "the static scratch must hold the largest chunk count rows_per_chunk() gives");
static __device__ __align__(256) float g_static_ln_scratch[kStaticLnChunks * kStaticLnMaxD * 2];

namespace {
std::mutex g_static_ln_mutex;
float* g_static_ln_ptr[64] = {nullptr};

// Device address of g_static_ln_scratch on the current device.
int static_ln_scratch(float** out) {
  int dev = 0;
  CIGN_CHECK_CUDA(cudaGetDevice(&dev), "dropout_ln_bwd_static: cudaGetDevice");
  CIGN_REQUIRE(dev >= 0 && dev < 64, CIGN_ERR_UNSUPPORTED,
               "dropout_ln_bwd_static: device id %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_static_ln_mutex);
  if (g_static_ln_ptr[dev] == nullptr) {
    void* p = nullptr;
    CIGN_CHECK_CUDA(cudaGetSymbolAddress(&p, g_static_ln_scratch),
                    "dropout_ln_bwd_static: cudaGetSymbolAddress");
    g_static_ln_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_static_ln_ptr[dev];
  return CIGN_OK;
}
}  // namespace

extern "C" int cign_dropout_ln_bwd_static(int64_t n, int64_t d, const float* grad_y,
                                          const float* x, const float* w, const float* mean,
                                          const float* rstd, float p, uint64_t seed,
                                          float* grad_x, float* grad_w, float* grad_b,
                                          cign_stream_t stream) {
  const bool v4 = d % 4 == 0 && aligned16(x) && aligned16(w) && aligned16(grad_y) &&
                  aligned16(grad_x);
  int rc = check_rows(n, d, v4, "dropout_ln_bwd_static");
  if (rc) return rc;
  CIGN_REQUIRE(d <= kStaticLnMaxD && num_chunks(n) <= kStaticLnChunks, CIGN_ERR_UNSUPPORTED,
               "dropout_ln_bwd_static: needs %lld x %lld partials, the static scratch holds "
               "%lld x %lld", (long long)num_chunks(n), (long long)d,
               (long long)kStaticLnChunks, (long long)kStaticLnMaxD);
  CIGN_REQUIRE(grad_w && grad_b, CIGN_ERR_NULL_POINTER, "dropout_ln_bwd_static: NULL param grad");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n == 0) {
    CIGN_CHECK_CUDA(cudaMemsetAsync(grad_w, 0, d * sizeof(float), s), "memset");
    CIGN_CHECK_CUDA(cudaMemsetAsync(grad_b, 0, d * sizeof(float), s), "memset");
    return CIGN_OK;
  }
  CIGN_REQUIRE(grad_y && x && w && mean && rstd && grad_x, CIGN_ERR_NULL_POINTER,
               "dropout_ln_bwd_static: NULL");
  float* wsf = nullptr;
  rc = static_ln_scratch(&wsf);
  if (rc) return rc;
  if (v4) {
    CIGN_ROW_DISPATCH(4, d / 4, return (launch_ln_bwd<0, V_, P_, L_>(n, d, grad_y, x, nullptr, w, mean, rstd, p, seed, grad_x, grad_w, grad_b, wsf, s)));
  }
  CIGN_ROW_DISPATCH(1, d, return (launch_ln_bwd<0, V_, P_, L_>(n, d, grad_y, x, nullptr, w, mean, rstd, p, seed, grad_x, grad_w, grad_b, wsf, s)));
  return CIGN_OK;
}
