// Clifford interaction pack family (old/new interaction, tanh/none outer,
// old/new alpha weighting, any hop count K <= 32), forward and backward.
//
// Reference kernels: fused_clifford_pack_ext/fused_clifford_pack_cuda.cu
// (K=3 old interaction, :22-152), the generic-K inline kernels
// (fused_clifford_pack.py:88-117; generic_engine/fused_clifford_cign_generic.py
// :58-87) and the switch/CIGN packs (generic_engine/
// fused_clifford_switch_pack_ext/fused_clifford_switch_pack_cuda.cu:22-368,
// whose CIGN copy drops the tanh).
//
// One group of LPR lanes owns one node row; each lane keeps its slice of
// H_norm/C_norm (and of the gradients) in registers while it walks the K
// hops, so the backward needs no atomics: grad_H/grad_C are summed over k
// in registers and grad_alpha[n,k] is one group reduction per hop.  The K
// propagated tensors are read through a pointer list, so the caller's
// per-hop outputs need no torch.stack copy.
#include <algorithm>

#include "common.cuh"
#include "pack_math.cuh"

namespace cign {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxK = 32;

struct CPtrs { const float* p[kMaxK]; };
struct MPtrs { float* p[kMaxK]; };

template <int VEC, int VPL, int LPR>
struct PackCfg {
  static constexpr int kGroups = kThreads / LPR;
  static constexpr int kTile = LPR * VPL * VEC;
};

template <int LPR>
__device__ __forceinline__ unsigned pack_group_mask() {
  return LPR == 32 ? kFullMask
                   : (((1u << LPR) - 1u) << ((threadIdx.x & 31) / LPR * LPR));
}


template <int VEC, int VPL, int LPR>
__global__ void __launch_bounds__(kThreads)
pack_fwd_kernel(int64_t n, int64_t D, int K, int interaction, int outer, int weighting,
                const float* __restrict__ Hn, const float* __restrict__ Cn, CPtrs P,
                int64_t ldp, const float* __restrict__ alpha, float* __restrict__ out) {
  using V = typename VecT<VEC>::type;
  using Cfg = PackCfg<VEC, VPL, LPR>;
  const int lig = threadIdx.x % LPR;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * Cfg::kGroups + threadIdx.x / LPR;
  if (row >= n) return;
  const int64_t ow = weighting == 0 ? 2 * D * K : 2 * D;
  for (int64_t f0 = 0; f0 < D; f0 += Cfg::kTile) {
    V h[VPL], c[VPL], accD[VPL], accW[VPL];
#pragma unroll
    for (int q = 0; q < VPL; ++q) {
      const int64_t d = f0 + static_cast<int64_t>(lig + q * LPR) * VEC;
      if (d < D) {
        h[q] = ld_vec<VEC>(Hn + row * D + d);
        c[q] = ld_vec<VEC>(Cn + row * D + d);
      } else {
        vzero(h[q]);
        vzero(c[q]);
      }
      vzero(accD[q]);
      vzero(accW[q]);
    }
    for (int k = 0; k < K; ++k) {
      const float a = alpha != nullptr ? __ldg(alpha + row * K + k) : 1.0f;
      const float* pk = P.p[k] + row * ldp;
#pragma unroll
      for (int q = 0; q < VPL; ++q) {
        const int64_t d = f0 + static_cast<int64_t>(lig + q * LPR) * VEC;
        if (d >= D) continue;
        const V th = ldg_vec<VEC>(pk + d);
        const V tc = ldg_vec<VEC>(pk + D + d);
        V ow_, od_;
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          float Dv, Wv;
          interact_fwd(vel(h[q], j) * vel(tc, j), vel(c[q], j) * vel(th, j), interaction, outer,
                       Dv, Wv);
          // explicit rounded products: never contracted into the hop sum
          // below, so every kernel forming the pack gives the same bits
          vel(ow_, j) = __fmul_rn(a, Wv);
          vel(od_, j) = __fmul_rn(a, Dv);
        }
        if (weighting == 0) {
          float* o = out + row * ow + static_cast<int64_t>(k) * 2 * D + d;
          st_vec(o, ow_);
          st_vec(o + D, od_);
        } else {
          vadd(accD[q], od_);
          vadd(accW[q], ow_);
        }
      }
    }
    if (weighting == 1) {
#pragma unroll
      for (int q = 0; q < VPL; ++q) {
        const int64_t d = f0 + static_cast<int64_t>(lig + q * LPR) * VEC;
        if (d < D) {
          st_vec(out + row * ow + d, accD[q]);
          st_vec(out + row * ow + D + d, accW[q]);
        }
      }
    }
  }
}

// The block's hop gate evaluated inside the pack forward
// (generic_engine/model_cign.py:721-749 feeding :817-925):
//   alpha = softmax_k([H + C | |H - C|] @ W^T + b)   (score mode "new"; [H | C] for "old")
// then the pack with that alpha; alpha [N, K] is also written for the
// backward.  One warp per node row (float4 slices, lane l owns columns
// 4l + 128q); H and C come from HBM once for both steps.
// The gate dots run in the order of hop_gate_fwd_kernel (columns
// increasing, x/y/z/w, the sum half before the difference half, then one
// warp sum) and the pack in the order of pack_fwd_kernel: alpha and the
// packed output equal those kernels' bit for bit.  Hop 0's propagated rows
// are read together with H and C and its interaction terms formed before
// the gate's reductions, so that load's latency hides behind the gate; the
// later hops re-read H and C (L1 hits) instead of holding them, which keeps
// the kernel at three CTAs per SM.
template <int K, int VPL, int WEIGHTING>
// D <= 512: <= 85 registers, 3 CTAs (24 rows) per SM; wider rows keep their
// registers (capping them would spill)
__global__ void __launch_bounds__(kThreads, VPL <= 4 ? 3 : 1)
gate_pack_fwd_kernel(int64_t n, int64_t D, int gate_mode, int interaction, int outer,
                     const float* __restrict__ Hn, const float* __restrict__ Cn,
                     CPtrs P, int64_t ldp, const float* __restrict__ W,
                     const float* __restrict__ b, float* __restrict__ alpha_out,
                     float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (kThreads / 32) + (threadIdx.x >> 5);
  if (row >= n) return;
  const int64_t D2 = 2 * D;
  const float* hr = Hn + row * D;
  const float* cr = Cn + row * D;
  // hop 0's interaction terms (before the alpha scaling): its propagated
  // rows are loaded with H and C and combined while the gate reduces
  float4 w0[VPL], d0[VPL];
  float dot[K];
#pragma unroll
  for (int k = 0; k < K; ++k) dot[k] = 0.0f;
  const float* p0 = P.p[0] + row * ldp;
#pragma unroll
  for (int q = 0; q < VPL; ++q) {
    const int64_t d = static_cast<int64_t>(lane + q * 32) * 4;
    if (d < D) {
      const float4 h = ldg_vec<4>(hr + d);
      const float4 c = ldg_vec<4>(cr + d);
      const float4 th = ldg_vec<4>(p0 + d);
      const float4 tc = ldg_vec<4>(p0 + D + d);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float Dv, Wv;
        interact_fwd(vel(h, j) * vel(tc, j), vel(c, j) * vel(th, j), interaction, outer, Dv, Wv);
        vel(w0[q], j) = Wv;
        vel(d0[q], j) = Dv;
      }
      float4 g0, g1;
      if (gate_mode == 1) {
        g0 = make_float4(h.x + c.x, h.y + c.y, h.z + c.z, h.w + c.w);
        g1 = make_float4(fabsf(h.x - c.x), fabsf(h.y - c.y), fabsf(h.z - c.z), fabsf(h.w - c.w));
      } else {
        g0 = h;
        g1 = c;
      }
#pragma unroll
      for (int k = 0; k < K; ++k) {
        const float4 wa = ldg_vec<4>(W + k * D2 + d);
        const float4 wb = ldg_vec<4>(W + k * D2 + D + d);
        float t = dot[k];
        t = fmaf(g0.x, wa.x, t); t = fmaf(g0.y, wa.y, t); t = fmaf(g0.z, wa.z, t); t = fmaf(g0.w, wa.w, t);
        t = fmaf(g1.x, wb.x, t); t = fmaf(g1.y, wb.y, t); t = fmaf(g1.z, wb.z, t); t = fmaf(g1.w, wb.w, t);
        dot[k] = t;
      }
    } else {
      vzero(w0[q]);
      vzero(d0[q]);
    }
  }
  float m = -INFINITY;
#pragma unroll
  for (int k = 0; k < K; ++k) {
    dot[k] = warp_sum(dot[k]) + __ldg(b + k);
    m = fmaxf(m, dot[k]);
  }
  float ssum = 0.0f;
#pragma unroll
  for (int k = 0; k < K; ++k) {
    dot[k] = expf(dot[k] - m);
    ssum += dot[k];
  }
#pragma unroll
  for (int k = 0; k < K; ++k) {
    dot[k] = dot[k] / ssum;  // alpha_k, on every lane
    if (lane == k) alpha_out[row * K + k] = dot[k];
  }
  const int64_t ow = WEIGHTING == 0 ? 2 * D * K : 2 * D;
  float4 accD[WEIGHTING == 1 ? VPL : 1], accW[WEIGHTING == 1 ? VPL : 1];
#pragma unroll
  for (int q = 0; q < (WEIGHTING == 1 ? VPL : 1); ++q) {
    vzero(accD[q]);
    vzero(accW[q]);
  }
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const float a = dot[k];
    const float* pk = P.p[k] + row * ldp;
#pragma unroll
    for (int q = 0; q < VPL; ++q) {
      const int64_t d = static_cast<int64_t>(lane + q * 32) * 4;
      if (d >= D) continue;
      float4 ow_, od_;
      if (k == 0) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          vel(ow_, j) = __fmul_rn(a, vel(w0[q], j));
          vel(od_, j) = __fmul_rn(a, vel(d0[q], j));
        }
      } else {
        // H and C again (this warp read them above: L1 hits), so a lane keeps
        // no copy of them across the gate
        const float4 h = ldg_vec<4>(hr + d);
        const float4 c = ldg_vec<4>(cr + d);
        const float4 th = ldg_vec<4>(pk + d);
        const float4 tc = ldg_vec<4>(pk + D + d);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float Dv, Wv;
          interact_fwd(vel(h, j) * vel(tc, j), vel(c, j) * vel(th, j), interaction, outer,
                       Dv, Wv);
          vel(ow_, j) = __fmul_rn(a, Wv);
          vel(od_, j) = __fmul_rn(a, Dv);
        }
      }
      if constexpr (WEIGHTING == 0) {
        float* o = out + row * ow + static_cast<int64_t>(k) * 2 * D + d;
        st_vec(o, ow_);
        st_vec(o + D, od_);
      } else {
        vadd(accD[q], od_);
        vadd(accW[q], ow_);
      }
    }
  }
  if constexpr (WEIGHTING == 1) {
#pragma unroll
    for (int q = 0; q < VPL; ++q) {
      const int64_t d = static_cast<int64_t>(lane + q * 32) * 4;
      if (d < D) {
        st_vec(out + row * ow + d, accD[q]);
        st_vec(out + row * ow + D + d, accW[q]);
      }
    }
  }
}

template <int K, int VPL>
int launch_gate_pack(int64_t n, int64_t D, int gate_mode, int interaction, int outer,
                     int weighting, const float* H, const float* C, const CPtrs& pl, int64_t ldp,
                     const float* W, const float* b, float* alpha, float* out, cudaStream_t s) {
  const int64_t grid = (n + kThreads / 32 - 1) / (kThreads / 32);
  if (weighting == 0)
    gate_pack_fwd_kernel<K, VPL, 0><<<static_cast<unsigned>(grid), kThreads, 0, s>>>(
        n, D, gate_mode, interaction, outer, H, C, pl, ldp, W, b, alpha, out);
  else
    gate_pack_fwd_kernel<K, VPL, 1><<<static_cast<unsigned>(grid), kThreads, 0, s>>>(
        n, D, gate_mode, interaction, outer, H, C, pl, ldp, W, b, alpha, out);
  CIGN_CHECK_LAUNCH("gate_pack_fwd_kernel");
  return CIGN_OK;
}

template <int K>
int launch_gate_pack_k(int64_t n, int64_t D, int gate_mode, int interaction, int outer,
                       int weighting, const float* H, const float* C, const CPtrs& pl,
                       int64_t ldp, const float* W, const float* b, float* alpha, float* out,
                       cudaStream_t s) {
  if (D <= 128)
    return launch_gate_pack<K, 1>(n, D, gate_mode, interaction, outer, weighting, H, C, pl, ldp, W, b, alpha, out, s);
  if (D <= 256)
    return launch_gate_pack<K, 2>(n, D, gate_mode, interaction, outer, weighting, H, C, pl, ldp, W, b, alpha, out, s);
  if (D <= 512)
    return launch_gate_pack<K, 4>(n, D, gate_mode, interaction, outer, weighting, H, C, pl, ldp, W, b, alpha, out, s);
  return launch_gate_pack<K, 8>(n, D, gate_mode, interaction, outer, weighting, H, C, pl, ldp, W, b, alpha, out, s);
}

template <int VEC, int VPL, int LPR>
__global__ void __launch_bounds__(kThreads)
pack_bwd_kernel(int64_t n, int64_t D, int K, int interaction, int outer, int weighting,
                const float* __restrict__ GO, const float* __restrict__ Hn,
                const float* __restrict__ Cn, CPtrs P, int64_t ldp,
                const float* __restrict__ alpha, float* __restrict__ GH,
                float* __restrict__ GC, MPtrs GP, int64_t ldgp, int accumulate_p,
                float* __restrict__ GA) {
  using V = typename VecT<VEC>::type;
  using Cfg = PackCfg<VEC, VPL, LPR>;
  const int lig = threadIdx.x % LPR;
  const unsigned gmask = pack_group_mask<LPR>();
  const int64_t row = static_cast<int64_t>(blockIdx.x) * Cfg::kGroups + threadIdx.x / LPR;
  if (row >= n) return;
  const int64_t ow = weighting == 0 ? 2 * D * K : 2 * D;
  for (int64_t f0 = 0; f0 < D; f0 += Cfg::kTile) {
    V h[VPL], c[VPL], gh[VPL], gc[VPL], goD[VPL], goW[VPL];
#pragma unroll
    for (int q = 0; q < VPL; ++q) {
      const int64_t d = f0 + static_cast<int64_t>(lig + q * LPR) * VEC;
      vzero(gh[q]);
      vzero(gc[q]);
      if (d < D) {
        h[q] = ld_vec<VEC>(Hn + row * D + d);
        c[q] = ld_vec<VEC>(Cn + row * D + d);
        if (weighting == 1) {
          goD[q] = ld_vec<VEC>(GO + row * ow + d);
          goW[q] = ld_vec<VEC>(GO + row * ow + D + d);
        }
      } else {
        vzero(h[q]);
        vzero(c[q]);
        vzero(goD[q]);
        vzero(goW[q]);
      }
    }
    for (int k = 0; k < K; ++k) {
      const float a = alpha != nullptr ? __ldg(alpha + row * K + k) : 1.0f;
      const float* pk = P.p[k] + row * ldp;
      float* gpk = GP.p[k] + row * ldgp;
      float ga = 0.0f;
#pragma unroll
      for (int q = 0; q < VPL; ++q) {
        const int64_t d = f0 + static_cast<int64_t>(lig + q * LPR) * VEC;
        if (d >= D) continue;
        const V th = ldg_vec<VEC>(pk + d);
        const V tc = ldg_vec<VEC>(pk + D + d);
        V gW, gD;
        if (weighting == 0) {
          const float* go = GO + row * ow + static_cast<int64_t>(k) * 2 * D + d;
          gW = ld_vec<VEC>(go);
          gD = ld_vec<VEC>(go + D);
        } else {
          gW = goW[q];
          gD = goD[q];
        }
        V gth, gtc;
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          const float hv = vel(h[q], j), cv = vel(c[q], j);
          const float thv = vel(th, j), tcv = vel(tc, j);
          const DW r = interact(hv * tcv, cv * thv, interaction, outer);
          const float gWo = vel(gW, j), gDo = vel(gD, j);
          ga += gWo * r.W + gDo * r.D;
          const float gWa = gWo * a, gDa = gDo * a;
          const float gbhr = gDa * r.dD_hr + gWa * r.dW_hr;
          const float gbrh = gDa * r.dD_rh + gWa * r.dW_rh;
          vel(gh[q], j) += gbhr * tcv;
          vel(gc[q], j) += gbrh * thv;
          vel(gth, j) = gbrh * cv;
          vel(gtc, j) = gbhr * hv;
        }
        if (accumulate_p) {
          vadd(gth, ld_vec<VEC>(gpk + d));
          vadd(gtc, ld_vec<VEC>(gpk + D + d));
        }
        st_vec(gpk + d, gth);
        st_vec(gpk + D + d, gtc);
      }
      if (GA != nullptr) {
#pragma unroll
        for (int o = LPR / 2; o > 0; o >>= 1) ga += __shfl_xor_sync(gmask, ga, o, LPR);
        if (lig == 0) {
          if (f0 == 0) GA[row * K + k] = ga;
          else GA[row * K + k] += ga;
        }
      }
    }
#pragma unroll
    for (int q = 0; q < VPL; ++q) {
      const int64_t d = f0 + static_cast<int64_t>(lig + q * LPR) * VEC;
      if (d < D) {
        st_vec(GH + row * D + d, gh[q]);
        st_vec(GC + row * D + d, gc[q]);
      }
    }
  }
}

#define CIGN_PACK_DISPATCH(VEC_, FV_, CALL)                                    \
  do {                                                                         \
    if ((FV_) <= 8) { constexpr int V_ = VEC_, P_ = 1, L_ = 8; CALL; }         \
    else if ((FV_) <= 16) { constexpr int V_ = VEC_, P_ = 1, L_ = 16; CALL; }  \
    else if ((FV_) <= 32) { constexpr int V_ = VEC_, P_ = 1, L_ = 32; CALL; }  \
    else if ((FV_) <= 64) { constexpr int V_ = VEC_, P_ = 2, L_ = 32; CALL; }  \
    else { constexpr int V_ = VEC_, P_ = 4, L_ = 32; CALL; }                   \
  } while (0)

// The backward keeps gh/gc/h/c/gradient tiles live across the hop loop; one
// vector per lane (looping over D in 128-float tiles) keeps it near 80
// registers, i.e. three resident CTAs per SM.
#define CIGN_PACK_BWD_DISPATCH(VEC_, FV_, CALL)                                \
  do {                                                                         \
    if ((FV_) <= 8) { constexpr int V_ = VEC_, P_ = 1, L_ = 8; CALL; }         \
    else if ((FV_) <= 16) { constexpr int V_ = VEC_, P_ = 1, L_ = 16; CALL; }  \
    else { constexpr int V_ = VEC_, P_ = 1, L_ = 32; CALL; }                   \
  } while (0)

template <int VEC, int VPL, int LPR>
int launch_fwd(int64_t n, int64_t D, int K, int inter, int outer, int weighting,
               const float* H, const float* C, const CPtrs& P, int64_t ldp,
               const float* alpha, float* out, cudaStream_t s) {
  using Cfg = PackCfg<VEC, VPL, LPR>;
  const int64_t grid = (n + Cfg::kGroups - 1) / Cfg::kGroups;
  CIGN_REQUIRE(grid < (1ll << 31), CIGN_ERR_UNSUPPORTED, "pack_fwd: too many rows");
  pack_fwd_kernel<VEC, VPL, LPR><<<static_cast<unsigned>(grid), kThreads, 0, s>>>(
      n, D, K, inter, outer, weighting, H, C, P, ldp, alpha, out);
  CIGN_CHECK_LAUNCH("pack_fwd_kernel");
  return CIGN_OK;
}

template <int VEC, int VPL, int LPR>
int launch_bwd(int64_t n, int64_t D, int K, int inter, int outer, int weighting,
               const float* GO, const float* H, const float* C, const CPtrs& P, int64_t ldp,
               const float* alpha, float* GH, float* GC, const MPtrs& GP, int64_t ldgp,
               int acc, float* GA, cudaStream_t s) {
  using Cfg = PackCfg<VEC, VPL, LPR>;
  const int64_t grid = (n + Cfg::kGroups - 1) / Cfg::kGroups;
  CIGN_REQUIRE(grid < (1ll << 31), CIGN_ERR_UNSUPPORTED, "pack_bwd: too many rows");
  pack_bwd_kernel<VEC, VPL, LPR><<<static_cast<unsigned>(grid), kThreads, 0, s>>>(
      n, D, K, inter, outer, weighting, GO, H, C, P, ldp, alpha, GH, GC, GP, ldgp, acc, GA);
  CIGN_CHECK_LAUNCH("pack_bwd_kernel");
  return CIGN_OK;
}

int check_modes(int64_t n, int64_t d, int k, int inter, int outer, int weighting,
                const char* name) {
  CIGN_REQUIRE(n >= 0 && d >= 1, CIGN_ERR_INVALID_ARGUMENT, "%s: bad sizes", name);
  CIGN_REQUIRE(k >= 1 && k <= kMaxK, CIGN_ERR_UNSUPPORTED, "%s: hop count must be in [1, %d]",
               name, kMaxK);
  CIGN_REQUIRE(inter == 0 || inter == 1, CIGN_ERR_INVALID_ARGUMENT,
               "%s: interaction must be 0 (old) or 1 (new)", name);
  CIGN_REQUIRE(outer == 0 || outer == 1, CIGN_ERR_INVALID_ARGUMENT,
               "%s: outer must be 0 (none) or 1 (tanh)", name);
  CIGN_REQUIRE(weighting == 0 || weighting == 1, CIGN_ERR_INVALID_ARGUMENT,
               "%s: weighting must be 0 (old) or 1 (new)", name);
  return CIGN_OK;
}

}  // namespace
}  // namespace cign

using namespace cign;

extern "C" {

int cign_pack_fwd(int64_t n, int64_t d, int32_t k, int32_t interaction, int32_t outer,
                  int32_t weighting, const float* H, const float* C, const float* const* P,
                  int64_t ldp, const float* alpha, float* out, cign_stream_t stream) {
  int rc = check_modes(n, d, k, interaction, outer, weighting, "pack_fwd");
  if (rc) return rc;
  if (n == 0) return CIGN_OK;
  CIGN_REQUIRE(H && C && P && out, CIGN_ERR_NULL_POINTER, "pack_fwd: NULL argument");
  CIGN_REQUIRE(ldp >= 2 * d, CIGN_ERR_INVALID_ARGUMENT, "pack_fwd: ldp < 2D");
  CPtrs pl{};
  bool v4 = d % 4 == 0 && ldp % 4 == 0 && aligned16(H) && aligned16(C) && aligned16(out);
  for (int i = 0; i < k; ++i) {
    CIGN_REQUIRE(P[i] != nullptr, CIGN_ERR_NULL_POINTER, "pack_fwd: P[%d] is NULL", i);
    pl.p[i] = P[i];
    v4 = v4 && aligned16(P[i]);
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (v4) {
    CIGN_PACK_DISPATCH(4, d / 4, return (launch_fwd<V_, P_, L_>(n, d, k, interaction, outer, weighting, H, C, pl, ldp, alpha, out, s)));
  }
  CIGN_PACK_DISPATCH(1, d, return (launch_fwd<V_, P_, L_>(n, d, k, interaction, outer, weighting, H, C, pl, ldp, alpha, out, s)));
  return CIGN_OK;
}

int cign_gate_pack_fwd(int64_t n, int64_t d, int32_t k, int32_t gate_mode,
                       int32_t interaction, int32_t outer, int32_t weighting, const float* H,
                       const float* C, const float* const* P, int64_t ldp, const float* gate_w,
                       const float* gate_b, float* alpha, float* out, cign_stream_t stream) {
  int rc = check_modes(n, d, k, interaction, outer, weighting, "gate_pack_fwd");
  if (rc) return rc;
  CIGN_REQUIRE(k >= 1 && k <= 8 && (gate_mode == 0 || gate_mode == 1), CIGN_ERR_UNSUPPORTED,
               "gate_pack_fwd: needs 1 <= K <= 8 and gate mode 0 or 1");
  CIGN_REQUIRE(d % 4 == 0 && d <= 1024 && ldp % 4 == 0, CIGN_ERR_UNSUPPORTED,
               "gate_pack_fwd: needs D %% 4 == 0, D <= 1024 and ldp %% 4 == 0");
  if (n == 0) return CIGN_OK;
  CIGN_REQUIRE(H && C && P && gate_w && gate_b && alpha && out, CIGN_ERR_NULL_POINTER,
               "gate_pack_fwd: NULL argument");
  CIGN_REQUIRE(ldp >= 2 * d, CIGN_ERR_INVALID_ARGUMENT, "gate_pack_fwd: ldp < 2D");
  CIGN_REQUIRE(aligned16(H) && aligned16(C) && aligned16(out) && aligned16(gate_w),
               CIGN_ERR_ALIGNMENT, "gate_pack_fwd: H, C, out and gate_w must be 16-byte aligned");
  CPtrs pl{};
  for (int i = 0; i < k; ++i) {
    CIGN_REQUIRE(P[i] != nullptr, CIGN_ERR_NULL_POINTER, "gate_pack_fwd: P[%d] is NULL", i);
    CIGN_REQUIRE(aligned16(P[i]), CIGN_ERR_ALIGNMENT, "gate_pack_fwd: P[%d] not 16-byte aligned",
                 i);
    pl.p[i] = P[i];
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (k) {
#define CIGN_GATE_PACK_K(KK) \
    case KK: return launch_gate_pack_k<KK>(n, d, gate_mode, interaction, outer, weighting, H, C, pl, ldp, gate_w, gate_b, alpha, out, s);
    CIGN_GATE_PACK_K(1) CIGN_GATE_PACK_K(2) CIGN_GATE_PACK_K(3) CIGN_GATE_PACK_K(4)
    CIGN_GATE_PACK_K(5) CIGN_GATE_PACK_K(6) CIGN_GATE_PACK_K(7) CIGN_GATE_PACK_K(8)
#undef CIGN_GATE_PACK_K
  }
  return CIGN_OK;
}

int cign_pack_bwd(int64_t n, int64_t d, int32_t k, int32_t interaction, int32_t outer,
                  int32_t weighting, const float* grad_out, const float* H, const float* C,
                  const float* const* P, int64_t ldp, const float* alpha, float* grad_H,
                  float* grad_C, float* const* grad_P, int64_t ldgp, int32_t accumulate_p,
                  float* grad_alpha, cign_stream_t stream) {
  int rc = check_modes(n, d, k, interaction, outer, weighting, "pack_bwd");
  if (rc) return rc;
  if (n == 0) return CIGN_OK;
  CIGN_REQUIRE(grad_out && H && C && P && grad_H && grad_C && grad_P, CIGN_ERR_NULL_POINTER,
               "pack_bwd: NULL argument");
  CIGN_REQUIRE(ldp >= 2 * d && ldgp >= 2 * d, CIGN_ERR_INVALID_ARGUMENT,
               "pack_bwd: ldp/ldgp < 2D");
  CPtrs pl{};
  MPtrs gl{};
  bool v4 = d % 4 == 0 && ldp % 4 == 0 && ldgp % 4 == 0 && aligned16(grad_out) &&
            aligned16(H) && aligned16(C) && aligned16(grad_H) && aligned16(grad_C);
  for (int i = 0; i < k; ++i) {
    CIGN_REQUIRE(P[i] != nullptr && grad_P[i] != nullptr, CIGN_ERR_NULL_POINTER,
                 "pack_bwd: P[%d]/grad_P[%d] is NULL", i, i);
    pl.p[i] = P[i];
    gl.p[i] = grad_P[i];
    v4 = v4 && aligned16(P[i]) && aligned16(grad_P[i]);
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (v4) {
    CIGN_PACK_BWD_DISPATCH(4, d / 4, return (launch_bwd<V_, P_, L_>(n, d, k, interaction, outer, weighting, grad_out, H, C, pl, ldp, alpha, grad_H, grad_C, gl, ldgp, accumulate_p, grad_alpha, s)));
  }
  CIGN_PACK_BWD_DISPATCH(1, d, return (launch_bwd<V_, P_, L_>(n, d, k, interaction, outer, weighting, grad_out, H, C, pl, ldp, alpha, grad_H, grad_C, gl, ldgp, accumulate_p, grad_alpha, s)));
  return CIGN_OK;
}

}  // extern "C"
