// Fixed-CSR SpMM and the k-hop propagation recurrence (forward P^p X and the
// transposed backward chain) for sm_100a.
//
// Design
//   * Row-split gather SpMM.  A group of LPR lanes (LPR = 8/16/32) owns one
//     output row and keeps the row's feature tile in registers (VPL vectors
//     of VEC floats per lane).  Column ids / values of the row are read
//     lane-parallel (coalesced) and broadcast with shuffles; each edge then
//     costs LPR*VPL vector loads of the neighbour's feature row, issued two
//     to four edges at a time for memory-level parallelism.  Rows wider than
//     one tile are split over the grid's second dimension (one feature tile
//     per block row), so the register footprint per lane, and with it the
//     number of resident warps, stays that of a 256-float row.
//     Measured on the cfg2 power-law graph this beat shared-memory staging
//     (cp.async rings, and TMA bulk copies per neighbour row, whose per-copy
//     cost put a ~95 us floor under every width) at every F.
//   * Power-law graphs have hub rows (thousands of non-zeros).  Rows with
//     more than kSegLen non-zeros are cut at plan time into segments of
//     kSegLen edges; every segment is one group's work item (scheduled
//     first), writing a partial tile to the workspace, and a combine kernel
//     sums each hub row's partials in segment order.  The work per group is
//     thus bounded by kSegLen edges and the result is deterministic.
//   * The backward "+ g" of the hop chain is the SpMM epilogue (addend).
//   * Reference: MultiHopCsrPlan (multihop_csr_ext/multihop_csr_pipeline_cuda.cu
//     :113-322) drives three cuSPARSE SpMMs plus two add kernels per call.
#include <cuda_bf16.h>

#include <algorithm>
#include <vector>

#include "common.cuh"

struct cign_spmm_plan {
  cign_csr_f32 p;
  cign_csr_f32 pt;
  bool pt_is_p;
  cign::SegList seg_p;
  cign::SegList seg_pt;  // unused (seg_p serves both) when pt_is_p
  int device;
};

namespace cign {
namespace {

// 4 warps (rows) per CTA: a CTA holds its SM slot until its longest row is
// done, and the power-law row lengths leave fewer idle warp slots behind
// with small CTAs (measured on the cfg2 graph: 118 us per F=1024 hop
// against 125 us at 8 warps per CTA; 2 warps gave the same as 4).
constexpr int kThreads = 128;
constexpr int kSegLen = 128;  // edges per work item of a hub row

template <int VEC, int VPL, int LPR>
struct SpmmCfg {
  static constexpr int kGroups = kThreads / LPR;        // groups per CTA
  static constexpr int kTile = LPR * VPL * VEC;         // floats per pass
  static constexpr int kUnroll = VPL >= 4 ? 2 : 4;      // edges in flight
};

// acc[q] += sum over edges e in {start, start+step, ...} < e1 of
//           val[e] * X[col[e] * ldx + xf0 + (lig + q*LPR)*VEC ...]
// (feature f0 + (lig + q*LPR)*VEC < F of the F-wide row; ldx = F and
// xf0 = f0 for a plain [*, F] X).  Edges are fetched LPR at a time (one per
// lane) and broadcast.
template <int VEC, int VPL, int LPR>
__device__ __forceinline__ void gather_edges(
    const int* __restrict__ col, const float* __restrict__ val, int start,
    int e1, int step, const float* __restrict__ X, int64_t ldx, int64_t xf0, int64_t F,
    int64_t f0, int lig, unsigned gmask, typename VecT<VEC>::type (&acc)[VPL]) {
  using V = typename VecT<VEC>::type;
  using Cfg = SpmmCfg<VEC, VPL, LPR>;
  for (int base = start; base < e1; base += step) {
    const int my = base + lig;
    int c = 0;
    float v = 0.0f;
    if (my < e1) {
      c = __ldg(col + my);
      v = __ldg(val + my);
    }
    const int cnt = min(LPR, e1 - base);
    int t = 0;
    for (; t + Cfg::kUnroll <= cnt; t += Cfg::kUnroll) {
      int cc[Cfg::kUnroll];
      float vv[Cfg::kUnroll];
#pragma unroll
      for (int u = 0; u < Cfg::kUnroll; ++u) {
        cc[u] = __shfl_sync(gmask, c, t + u, LPR);
        vv[u] = __shfl_sync(gmask, v, t + u, LPR);
      }
      V xv[Cfg::kUnroll][VPL];
#pragma unroll
      for (int u = 0; u < Cfg::kUnroll; ++u) {
        const float* xr = X + static_cast<int64_t>(cc[u]) * ldx + xf0;
#pragma unroll
        for (int q = 0; q < VPL; ++q) {
          const int64_t fi = static_cast<int64_t>(lig + q * LPR) * VEC;
          if (f0 + fi < F) xv[u][q] = ldg_vec<VEC>(xr + fi);
          else vzero(xv[u][q]);
        }
      }
#pragma unroll
      for (int u = 0; u < Cfg::kUnroll; ++u)
#pragma unroll
        for (int q = 0; q < VPL; ++q) vfma(acc[q], vv[u], xv[u][q]);
    }
    for (; t < cnt; ++t) {
      const int c0 = __shfl_sync(gmask, c, t, LPR);
      const float v0 = __shfl_sync(gmask, v, t, LPR);
      const float* xr = X + static_cast<int64_t>(c0) * ldx + xf0;
#pragma unroll
      for (int q = 0; q < VPL; ++q) {
        const int64_t fi = static_cast<int64_t>(lig + q * LPR) * VEC;
        if (f0 + fi < F) vfma(acc[q], v0, ldg_vec<VEC>(xr + fi));
      }
    }
  }
}

// Blocks [0, seg_blocks) process hub-row segments (one group each) into
// `partial`; the remaining blocks process the whole rows of at most kSegLen
// non-zeros, taken from the plan's length-ordered list `light` (n_light
// entries, longest first).  X is [rows of X, F] -- or, with X1 != NULL, the two column
// blocks [X | X1] of widths split and F - split held as separate row-major
// matrices (split a multiple of the tile width, so a tile lies in one).
template <int VEC, int VPL, int LPR, bool SPLIT = false>
__global__ void __launch_bounds__(kThreads)
spmm_rows_kernel(int n_light, const int* __restrict__ light, const int* __restrict__ crow,
                 const int* __restrict__ col, const float* __restrict__ val,
                 const int* __restrict__ seg_begin, const int* __restrict__ seg_end, int n_seg,
                 int seg_blocks, const float* __restrict__ X, int64_t F,
                 const float* __restrict__ X1,
                 int64_t split, const float* __restrict__ addend,
                 float* __restrict__ Y, float* __restrict__ partial) {
  using V = typename VecT<VEC>::type;
  using Cfg = SpmmCfg<VEC, VPL, LPR>;
  const int lig = threadIdx.x % LPR;
  const int group = threadIdx.x / LPR;
  const unsigned gmask =
      LPR == 32 ? kFullMask
                : (((1u << LPR) - 1u) << ((threadIdx.x & 31) / LPR * LPR));

  // one feature tile per block row of the grid (gridDim.y * kTile >= F)
  const int64_t f0 = static_cast<int64_t>(blockIdx.y) * Cfg::kTile;
  // the gathered matrix, its row stride and this tile's first column in it
  const float* Xg = X;
  int64_t ldx = F, xf0 = f0;
  if constexpr (SPLIT) {
    const bool second = f0 >= split;
    Xg = second ? X1 : X;
    ldx = second ? F - split : split;
    xf0 = second ? f0 - split : f0;
  }
  V acc[VPL];
#pragma unroll
  for (int q = 0; q < VPL; ++q) vzero(acc[q]);
  if (static_cast<int>(blockIdx.x) < seg_blocks) {
    const int64_t sidx = static_cast<int64_t>(blockIdx.x) * Cfg::kGroups + group;
    if (sidx >= n_seg) return;
    gather_edges<VEC, VPL, LPR>(col, val, seg_begin[sidx], seg_end[sidx], LPR, Xg, ldx, xf0, F,
                                f0, lig, gmask, acc);
    float* pr = partial + sidx * F;
#pragma unroll
    for (int q = 0; q < VPL; ++q) {
      const int64_t fi = static_cast<int64_t>(lig + q * LPR) * VEC;
      if (f0 + fi < F) st_vec(pr + f0 + fi, acc[q]);
    }
    return;
  }

  const int64_t item = static_cast<int64_t>(blockIdx.x - seg_blocks) * Cfg::kGroups + group;
  if (item >= n_light) return;
  const int64_t row64 = light[item];  // at most kSegLen non-zeros
  const int e0 = crow[row64];
  const int e1 = crow[row64 + 1];
  gather_edges<VEC, VPL, LPR>(col, val, e0, e1, LPR, Xg, ldx, xf0, F, f0, lig, gmask, acc);
  float* yr = Y + row64 * F + f0;
  const float* ar = addend != nullptr ? addend + row64 * F + f0 : nullptr;
#pragma unroll
  for (int q = 0; q < VPL; ++q) {
    const int64_t fi = static_cast<int64_t>(lig + q * LPR) * VEC;
    if (f0 + fi < F) {
      if (ar != nullptr) vadd(acc[q], ld_vec<VEC>(ar + fi));
      st_vec(yr + fi, acc[q]);
    }
  }
}

// Hub-row combine: Y[row] = sum of the row's segment partials (+ addend).
// Block (hub, chunk) covers kCombineThreads * VEC columns of one hub row; its
// kCombineWays thread rows each sum a contiguous quarter of the segments in
// order (several loads in flight), and the quarter sums are then added in
// quarter order -- a fixed order, with a critical path a quarter as long.
constexpr int kCombineThreads = 64;
constexpr int kCombineWays = 4;

// OUT_BF16: Y is bf16 (VEC == 4), each sum rounded to nearest even.
template <int VEC, bool OUT_BF16 = false>
__global__ void __launch_bounds__(kCombineThreads * kCombineWays)
spmm_combine_kernel(const int* __restrict__ heavy_row, const int* __restrict__ heavy_first,
                    const float* __restrict__ partial, int64_t F,
                    const float* __restrict__ addend, void* __restrict__ Y) {
  using V = typename VecT<VEC>::type;
  __shared__ V part[kCombineWays - 1][kCombineThreads];
  const int h = blockIdx.x;
  const int tx = threadIdx.x % kCombineThreads, way = threadIdx.x / kCombineThreads;
  const int64_t f = (static_cast<int64_t>(blockIdx.y) * kCombineThreads + tx) * VEC;
  const int s0 = heavy_first[h], s1 = heavy_first[h + 1];
  const int per = (s1 - s0 + kCombineWays - 1) / kCombineWays;
  const int a = min(s1, s0 + way * per), b = min(s1, a + per);
  V acc;
  vzero(acc);
  if (f < F) acc = ordered_sum<VEC>(partial + f, F, a, b);
  if (way > 0) part[way - 1][tx] = acc;
  __syncthreads();
  if (way > 0 || f >= F) return;
#pragma unroll
  for (int w = 0; w < kCombineWays - 1; ++w) vadd(acc, part[w][tx]);
  const int64_t row = heavy_row[h];
  if (addend != nullptr) vadd(acc, ld_vec<VEC>(addend + row * F + f));
  if constexpr (OUT_BF16) {
    static_assert(VEC == 4, "bf16 combine stores 4 values per thread");
    __nv_bfloat162* y = reinterpret_cast<__nv_bfloat162*>(static_cast<__nv_bfloat16*>(Y) + row * F + f);
    y[0] = __floats2bfloat162_rn(vel(acc, 0), vel(acc, 1));
    y[1] = __floats2bfloat162_rn(vel(acc, 2), vel(acc, 3));
  } else {
    st_vec(static_cast<float*>(Y) + row * F + f, acc);
  }
}

template <int VEC, bool OUT_BF16 = false>
int launch_spmm_combine(const SegList& sl, const float* partial, int64_t F, const float* addend,
                        void* Y, cudaStream_t stream) {
  if (sl.n_heavy == 0) return CIGN_OK;
  const int64_t per_block = static_cast<int64_t>(kCombineThreads) * VEC;
  const int64_t chunks = (F / VEC * VEC + per_block - 1) / per_block;
  CIGN_REQUIRE(chunks < 65536, CIGN_ERR_UNSUPPORTED, "spmm: F too large for the hub combine");
  const dim3 grid(static_cast<unsigned>(sl.n_heavy), static_cast<unsigned>(chunks));
  spmm_combine_kernel<VEC, OUT_BF16><<<grid, kCombineThreads * kCombineWays, 0, stream>>>(
      sl.heavy_row(), sl.heavy_first(), partial, F, addend, Y);
  CIGN_CHECK_LAUNCH("spmm_combine_kernel");
  return CIGN_OK;
}

// ------------------------------------------------------ bf16 storage
// The same row-split gather over bf16 feature rows (storage precision of
// the large-graph configuration: bf16 features, fp32 accumulation).  Lane l
// loads 16 bytes = 8 bf16 per vector, widens them to fp32 and accumulates
// in fp32 in the same edge order as the fp32 kernel; the output row is
// stored as fp32 or rounded (to nearest even) to bf16.  A warp owns one
// row's tile of 32 * VPL * 8 features (1 KB of bf16 per edge at VPL = 2),
// UNROLL edges' loads in flight.  Hub segments write fp32 partials that the
// fp32 path's combine sums (in its order) and stores as fp32 or bf16.
__device__ __forceinline__ void bf8_to_f32(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(b[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ uint4 f32_to_bf8(const float (&f)[8]) {
  uint4 u;
  __nv_bfloat162* b = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) b[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return u;
}

template <int VPL, bool OUT_BF16, int UNROLL>
__global__ void __launch_bounds__(kThreads)
spmm_rows_bf16_kernel(int rows, const int* __restrict__ crow, const int* __restrict__ col,
                      const float* __restrict__ val, const int* __restrict__ seg_begin,
                      const int* __restrict__ seg_end, int n_seg, int seg_blocks,
                      const __nv_bfloat16* __restrict__ X, int64_t F, void* __restrict__ Y,
                      float* __restrict__ partial) {
  constexpr int kTile = 32 * VPL * 8;
  const int lane = threadIdx.x & 31;
  const int group = threadIdx.x >> 5;
  const int64_t f0 = static_cast<int64_t>(blockIdx.y) * kTile;
  int64_t item;
  int e0, e1;
  bool seg;
  if (static_cast<int>(blockIdx.x) < seg_blocks) {
    item = static_cast<int64_t>(blockIdx.x) * (kThreads / 32) + group;
    if (item >= n_seg) return;
    e0 = seg_begin[item];
    e1 = seg_end[item];
    seg = true;
  } else {
    item = static_cast<int64_t>(blockIdx.x - seg_blocks) * (kThreads / 32) + group;
    if (item >= rows) return;
    e0 = crow[item];
    e1 = crow[item + 1];
    if (e1 - e0 > kSegLen) return;  // a hub row: done by segments + combine
    seg = false;
  }
  float acc[VPL][8];
#pragma unroll
  for (int q = 0; q < VPL; ++q)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[q][j] = 0.0f;
  for (int base = e0; base < e1; base += 32) {
    const int my = base + lane;
    int c = 0;
    float v = 0.0f;
    if (my < e1) {
      c = __ldg(col + my);
      v = __ldg(val + my);
    }
    const int cnt = min(32, e1 - base);
    for (int t = 0; t < cnt; t += UNROLL) {
      uint4 xv[UNROLL][VPL];
      float vv[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const bool on = t + u < cnt;
        // (t, u and cnt are warp-uniform: every lane takes the same branch)
        const int cc = __shfl_sync(kFullMask, c, on ? t + u : 0);
        const float vu = __shfl_sync(kFullMask, v, on ? t + u : 0);
        vv[u] = on ? vu : 0.0f;
        const __nv_bfloat16* xr = X + static_cast<int64_t>(cc) * F;
#pragma unroll
        for (int q = 0; q < VPL; ++q) {
          const int64_t fi = f0 + static_cast<int64_t>(lane + q * 32) * 8;
          xv[u][q] = (on && fi < F) ? __ldg(reinterpret_cast<const uint4*>(xr + fi))
                                    : make_uint4(0u, 0u, 0u, 0u);
        }
      }
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        if (t + u >= cnt) break;
#pragma unroll
        for (int q = 0; q < VPL; ++q) {
          float xf[8];
          bf8_to_f32(xv[u][q], xf);
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[q][j] = fmaf(vv[u], xf[j], acc[q][j]);
        }
      }
    }
  }
#pragma unroll
  for (int q = 0; q < VPL; ++q) {
    const int64_t fi = f0 + static_cast<int64_t>(lane + q * 32) * 8;
    if (fi >= F) continue;
    if (seg) {
      float* pr = partial + item * F + fi;
      st_vec(pr, make_float4(acc[q][0], acc[q][1], acc[q][2], acc[q][3]));
      st_vec(pr + 4, make_float4(acc[q][4], acc[q][5], acc[q][6], acc[q][7]));
    } else if (OUT_BF16) {
      *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(Y) + item * F + fi) =
          f32_to_bf8(acc[q]);
    } else {
      float* yr = static_cast<float*>(Y) + item * F + fi;
      st_vec(yr, make_float4(acc[q][0], acc[q][1], acc[q][2], acc[q][3]));
      st_vec(yr + 4, make_float4(acc[q][4], acc[q][5], acc[q][6], acc[q][7]));
    }
  }
}

template <int VPL, bool OUT_BF16, int UNROLL = 4>
int launch_spmm_bf16_cfg(const cign_csr_f32& m, const SegList& sl, const __nv_bfloat16* X,
                         int64_t F, void* Y, float* partial, cudaStream_t stream) {
  constexpr int kTile = 32 * VPL * 8;
  const int64_t seg_blocks = (sl.n_seg + kThreads / 32 - 1) / (kThreads / 32);
  const int64_t grid = seg_blocks + (m.rows + kThreads / 32 - 1) / (kThreads / 32);
  if (grid == 0) return CIGN_OK;
  const int64_t tiles = (F + kTile - 1) / kTile;
  CIGN_REQUIRE(grid < (1ll << 31) && tiles <= 65535, CIGN_ERR_UNSUPPORTED,
               "spmm_bf16: grid too large");
  spmm_rows_bf16_kernel<VPL, OUT_BF16, UNROLL>
      <<<dim3(static_cast<unsigned>(grid), static_cast<unsigned>(tiles)), kThreads, 0, stream>>>(
          static_cast<int>(m.rows), m.crow, m.col, m.val, sl.seg_begin(), sl.seg_end(),
          static_cast<int>(sl.n_seg), static_cast<int>(seg_blocks), X, F, Y, partial);
  CIGN_CHECK_LAUNCH("spmm_rows_bf16_kernel");
  // hub rows: the fp32 path's combine (same segment sums, same order)
  return launch_spmm_combine<4, OUT_BF16>(sl, partial, F, nullptr, Y, stream);
}

int run_spmm_bf16(const cign_spmm_plan* plan, int transpose, const __nv_bfloat16* X, int64_t F,
                  void* Y, bool y_bf16, float* partial, cudaStream_t s) {
  const bool use_t = transpose != 0 && !plan->pt_is_p;
  const cign_csr_f32& m = use_t ? plan->pt : plan->p;
  const SegList& sl = use_t ? plan->seg_pt : plan->seg_p;
  if (F <= 256) {
    return y_bf16 ? launch_spmm_bf16_cfg<1, true>(m, sl, X, F, Y, partial, s)
                  : launch_spmm_bf16_cfg<1, false>(m, sl, X, F, Y, partial, s);
  }
  // 512-feature tiles (1 KB per edge), two edges' loads in flight (48
  // registers): measured faster than four in flight (80 registers), 256- and
  // 1024-feature tiles on the cfg2 graph and on a cfg5 row block
  return y_bf16 ? launch_spmm_bf16_cfg<2, true, 2>(m, sl, X, F, Y, partial, s)
                : launch_spmm_bf16_cfg<2, false, 2>(m, sl, X, F, Y, partial, s);
}

// Plan-time validation of a CSR: crow monotone with crow[0]=0, crow[rows]=nnz,
// all columns in range.  Sets *bad to 1 on the first violation.
__global__ void csr_validate_kernel(int64_t rows, int64_t cols, int64_t nnz,
                                    const int* __restrict__ crow,
                                    const int* __restrict__ col,
                                    int* __restrict__ bad) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       i < rows; i += stride) {
    if (crow[i] > crow[i + 1]) atomicExch(bad, 1);
  }
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       e < nnz; e += stride) {
    const int c = col[e];
    if (c < 0 || c >= cols) atomicExch(bad, 1);
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    if (crow[0] != 0 || static_cast<int64_t>(crow[rows]) != nnz)
      atomicExch(bad, 1);
  }
}

template <int VEC, int VPL, int LPR>
int launch_spmm_cfg(const cign_csr_f32& m, const SegList& sl, const float* X, int64_t F,
                    const float* addend, float* Y, float* partial, cudaStream_t stream,
                    const float* X1 = nullptr, int64_t split = 0) {
  using Cfg = SpmmCfg<VEC, VPL, LPR>;
  const int64_t seg_blocks = (sl.n_seg + Cfg::kGroups - 1) / Cfg::kGroups;
  const int64_t light_blocks = (sl.n_light + Cfg::kGroups - 1) / Cfg::kGroups;
  const int64_t grid = seg_blocks + light_blocks;
  if (grid == 0) return CIGN_OK;
  CIGN_REQUIRE(grid < (1ll << 31), CIGN_ERR_UNSUPPORTED, "spmm: grid too large");
  // one feature tile per block row of the grid
  const int64_t tiles = (F + Cfg::kTile - 1) / Cfg::kTile;
  CIGN_REQUIRE(tiles <= 65535, CIGN_ERR_UNSUPPORTED, "spmm: F too large (%lld tiles)",
               static_cast<long long>(tiles));
  const dim3 g(static_cast<unsigned>(grid), static_cast<unsigned>(tiles));
  if (X1 != nullptr)
    spmm_rows_kernel<VEC, VPL, LPR, true><<<g, kThreads, 0, stream>>>(
        static_cast<int>(sl.n_light), sl.light_row(), m.crow, m.col, m.val, sl.seg_begin(),
        sl.seg_end(), static_cast<int>(sl.n_seg), static_cast<int>(seg_blocks), X, F, X1, split,
        addend, Y, partial);
  else
    spmm_rows_kernel<VEC, VPL, LPR, false><<<g, kThreads, 0, stream>>>(
        static_cast<int>(sl.n_light), sl.light_row(), m.crow, m.col, m.val, sl.seg_begin(),
        sl.seg_end(), static_cast<int>(sl.n_seg), static_cast<int>(seg_blocks), X, F, nullptr, 0,
        addend, Y, partial);
  CIGN_CHECK_LAUNCH("spmm_rows_kernel");
  return launch_spmm_combine<VEC>(sl, partial, F, addend, Y, stream);
}

template <int VEC>
int launch_spmm_vec(const cign_csr_f32& m, const SegList& sl, const float* X, int64_t F,
                    const float* addend, float* Y, float* partial, cudaStream_t stream) {
  const int64_t fv = F / VEC;  // vectors per row
  if (fv <= 8) return launch_spmm_cfg<VEC, 1, 8>(m, sl, X, F, addend, Y, partial, stream);
  if (fv <= 16) return launch_spmm_cfg<VEC, 1, 16>(m, sl, X, F, addend, Y, partial, stream);
  if (fv <= 32) return launch_spmm_cfg<VEC, 1, 32>(m, sl, X, F, addend, Y, partial, stream);
  if (fv <= 64) return launch_spmm_cfg<VEC, 2, 32>(m, sl, X, F, addend, Y, partial, stream);
  // wider float4 rows: 256-float tiles over the grid's second dimension keep
  // the register footprint (and so the warps in flight, four edges' loads
  // each) of the narrow case.  Measured on the cfg2 graph this beat 512- and
  // 1024-float tiles, deeper unrolling, persistent warps striding over
  // (tile, row) items, lane-private cp.async rings of 4-12 rows and L2
  // evict-last / evict-first hints: every variant gathers at or below
  // ~13 TB/s of neighbour rows, the L2-to-SM ceiling of this access pattern.
  if (VEC == 4) return launch_spmm_cfg<VEC, 2, 32>(m, sl, X, F, addend, Y, partial, stream);
  if (fv <= 128) return launch_spmm_cfg<VEC, 4, 32>(m, sl, X, F, addend, Y, partial, stream);
  return launch_spmm_cfg<VEC, 8, 32>(m, sl, X, F, addend, Y, partial, stream);
}

// Workspace of one SpMM: hub-row partials [n_seg, F] (+ 256 bytes of
// alignment slack).
size_t partial_bytes(const cign_spmm_plan* plan, int64_t F) {
  const int64_t n = std::max(plan->seg_p.n_seg, plan->pt_is_p ? 0 : plan->seg_pt.n_seg);
  return (static_cast<size_t>(n) * F * sizeof(float) + 255) / 256 * 256 + 256;
}

int run_spmm(const cign_spmm_plan* plan, int transpose, const float* X, int64_t F,
             const float* addend, float* Y, float* partial, cudaStream_t stream) {
  const bool use_t = transpose != 0 && !plan->pt_is_p;
  const cign_csr_f32& m = use_t ? plan->pt : plan->p;
  const SegList& sl = use_t ? plan->seg_pt : plan->seg_p;
  const bool vec4 = (F % 4 == 0) && aligned16(X) && aligned16(Y) && aligned16(partial) &&
                    (addend == nullptr || aligned16(addend));
  if (vec4) return launch_spmm_vec<4>(m, sl, X, F, addend, Y, partial, stream);
  return launch_spmm_vec<1>(m, sl, X, F, addend, Y, partial, stream);
}

int check_csr_args(const cign_csr_f32* m, const char* name) {
  CIGN_REQUIRE(m != nullptr, CIGN_ERR_NULL_POINTER, "%s: csr is NULL", name);
  CIGN_REQUIRE(m->rows >= 0 && m->cols >= 0 && m->nnz >= 0,
               CIGN_ERR_INVALID_ARGUMENT, "%s: negative size", name);
  CIGN_REQUIRE(m->rows < (1ll << 31) && m->cols < (1ll << 31) &&
                   m->nnz < (1ll << 31),
               CIGN_ERR_UNSUPPORTED, "%s: int32 CSR limits exceeded", name);
  CIGN_REQUIRE(m->crow != nullptr, CIGN_ERR_NULL_POINTER, "%s: crow is NULL", name);
  CIGN_REQUIRE(m->nnz == 0 || (m->col != nullptr && m->val != nullptr),
               CIGN_ERR_NULL_POINTER, "%s: col/val is NULL", name);
  return CIGN_OK;
}

// Validates the CSR on the device, then builds the hub-row segment list
// (device buffer owned by the plan).
int build_plan_segments(const cign_csr_f32& m, SegList* out) {
  int* bad_d = nullptr;
  CIGN_CHECK_CUDA(cudaMalloc(&bad_d, sizeof(int)), "plan: cudaMalloc");
  cudaMemset(bad_d, 0, sizeof(int));
  const int64_t work = std::max<int64_t>(std::max<int64_t>(m.rows, m.nnz), 1);
  const int blocks = static_cast<int>(std::min<int64_t>((work + 255) / 256, 4096));
  csr_validate_kernel<<<blocks, 256>>>(m.rows, m.cols, m.nnz, m.crow, m.col, bad_d);
  cudaError_t le = cudaGetLastError();
  int bad = 0;
  cudaError_t ce = cudaMemcpy(&bad, bad_d, sizeof(int), cudaMemcpyDeviceToHost);
  cudaFree(bad_d);
  if (le != cudaSuccess || ce != cudaSuccess)
    return set_error(CIGN_ERR_CUDA, "plan: csr validation failed: %s",
                     cudaGetErrorString(le != cudaSuccess ? le : ce));
  CIGN_REQUIRE(bad == 0, CIGN_ERR_INVALID_ARGUMENT,
               "plan: malformed CSR (crow not monotone from 0 to nnz, or a "
               "column index out of range)");
  return build_segments(m.crow, m.rows, kSegLen, out);
}

int check_dense(const cign_spmm_plan* plan, const float* X, int64_t F,
                const void* Y, const char* name, bool square = true) {
  CIGN_REQUIRE(plan != nullptr, CIGN_ERR_NULL_POINTER, "%s: plan is NULL", name);
  CIGN_REQUIRE(F > 0, CIGN_ERR_INVALID_ARGUMENT, "%s: F must be positive", name);
  CIGN_REQUIRE(!square || plan->p.rows == plan->p.cols, CIGN_ERR_INVALID_ARGUMENT,
               "%s: operator must be square", name);
  if (plan->p.rows > 0 || plan->p.cols > 0) {
    CIGN_REQUIRE(X != nullptr && Y != nullptr, CIGN_ERR_NULL_POINTER,
                 "%s: dense operand is NULL", name);
  }
  return CIGN_OK;
}

}  // namespace
}  // namespace cign

using namespace cign;

extern "C" {

int cign_spmm_plan_create(const cign_csr_f32* p, const cign_csr_f32* pt,
                          cign_spmm_plan** out) {
  CIGN_REQUIRE(out != nullptr, CIGN_ERR_NULL_POINTER, "plan_create: out is NULL");
  *out = nullptr;
  int rc = check_csr_args(p, "plan_create(P)");
  if (rc) return rc;
  const bool pt_is_p = pt == nullptr ||
                       (pt->crow == p->crow && pt->col == p->col && pt->val == p->val);
  if (!pt_is_p) {
    rc = check_csr_args(pt, "plan_create(P^T)");
    if (rc) return rc;
    CIGN_REQUIRE(pt->rows == p->cols && pt->cols == p->rows && pt->nnz == p->nnz,
                 CIGN_ERR_INVALID_ARGUMENT, "plan_create: P^T shape mismatch");
  }
  cign_spmm_plan* plan = new cign_spmm_plan();
  plan->p = *p;
  plan->pt = pt_is_p ? *p : *pt;
  plan->pt_is_p = pt_is_p;
  cudaGetDevice(&plan->device);
  rc = build_plan_segments(plan->p, &plan->seg_p);
  if (rc == CIGN_OK && !pt_is_p) rc = build_plan_segments(plan->pt, &plan->seg_pt);
  if (rc != CIGN_OK) {
    free_segments(&plan->seg_p);
    free_segments(&plan->seg_pt);
    delete plan;
    return rc;
  }
  *out = plan;
  clear_error();
  return CIGN_OK;
}

int cign_spmm_plan_destroy(cign_spmm_plan* plan) {
  if (plan == nullptr) return CIGN_OK;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(plan->device);
  free_segments(&plan->seg_p);
  free_segments(&plan->seg_pt);
  cudaSetDevice(prev);
  delete plan;
  return CIGN_OK;
}

int cign_spmm_plan_get_info(const cign_spmm_plan* plan, cign_spmm_plan_info* info) {
  CIGN_REQUIRE(plan != nullptr && info != nullptr, CIGN_ERR_NULL_POINTER,
               "plan_get_info: NULL argument");
  const SegList& t = plan->pt_is_p ? plan->seg_p : plan->seg_pt;
  info->rows = plan->p.rows;
  info->nnz = plan->p.nnz;
  info->heavy_rows = plan->seg_p.n_heavy;
  info->heavy_rows_t = t.n_heavy;
  info->segments = plan->seg_p.n_seg;
  info->segments_t = t.n_seg;
  info->max_degree = plan->seg_p.max_len;
  info->max_degree_t = t.max_len;
  info->segment_length = kSegLen;
  info->transpose_is_forward = plan->pt_is_p ? 1 : 0;
  return CIGN_OK;
}

size_t cign_spmm_workspace_bytes(const cign_spmm_plan* plan, int64_t F) {
  if (plan == nullptr || F <= 0) return 0;
  return partial_bytes(plan, F);
}

int cign_spmm(const cign_spmm_plan* plan, int transpose, const float* X, int64_t F,
              const float* addend, float* Y, void* ws, size_t ws_bytes,
              cign_stream_t stream) {
  int rc = check_dense(plan, X, F, Y, "spmm", false);
  if (rc) return rc;
  CIGN_REQUIRE(!(transpose && plan->pt_is_p && plan->p.rows != plan->p.cols),
               CIGN_ERR_INVALID_ARGUMENT,
               "spmm: a rectangular P needs its transpose at plan creation");
  CIGN_REQUIRE(X != Y || plan->p.rows == 0, CIGN_ERR_INVALID_ARGUMENT,
               "spmm: Y must not alias X");
  const size_t need = partial_bytes(plan, F);
  CIGN_REQUIRE(ws_bytes >= need && (need == 0 || ws != nullptr), CIGN_ERR_INVALID_ARGUMENT,
               "spmm: workspace too small (%zu < %zu bytes)", ws_bytes, need);
  return run_spmm(plan, transpose, X, F, addend, Y, static_cast<float*>(ws),
                  static_cast<cudaStream_t>(stream));
}

int cign_spmm_bf16(const cign_spmm_plan* plan, int transpose, const void* X, int64_t F, void* Y,
                   int y_bf16, void* ws, size_t ws_bytes, cign_stream_t stream) {
  int rc = check_dense(plan, static_cast<const float*>(X), F, Y, "spmm_bf16", false);
  if (rc) return rc;
  CIGN_REQUIRE(!(transpose && plan->pt_is_p && plan->p.rows != plan->p.cols),
               CIGN_ERR_INVALID_ARGUMENT,
               "spmm_bf16: a rectangular P needs its transpose at plan creation");
  CIGN_REQUIRE(F % 8 == 0, CIGN_ERR_UNSUPPORTED, "spmm_bf16: F must be a multiple of 8");
  CIGN_REQUIRE(aligned16(X) && aligned16(Y) && aligned16(ws), CIGN_ERR_ALIGNMENT,
               "spmm_bf16: X, Y and ws must be 16-byte aligned");
  CIGN_REQUIRE(X != Y || plan->p.rows == 0, CIGN_ERR_INVALID_ARGUMENT,
               "spmm_bf16: Y must not alias X");
  const size_t need = partial_bytes(plan, F);
  CIGN_REQUIRE(ws_bytes >= need && (need == 0 || ws != nullptr), CIGN_ERR_INVALID_ARGUMENT,
               "spmm_bf16: workspace too small (%zu < %zu bytes)", ws_bytes, need);
  return run_spmm_bf16(plan, transpose, static_cast<const __nv_bfloat16*>(X), F, Y, y_bf16 != 0,
                       static_cast<float*>(ws), static_cast<cudaStream_t>(stream));
}

int cign_multihop_fwd_bf16(const cign_spmm_plan* plan, int max_power, const void* X, int64_t F,
                           void* const* Y, void* ws, size_t ws_bytes, cign_stream_t stream) {
  CIGN_REQUIRE(max_power >= 1, CIGN_ERR_INVALID_ARGUMENT,
               "multihop_fwd_bf16: max_power must be >= 1");
  CIGN_REQUIRE(Y != nullptr, CIGN_ERR_NULL_POINTER, "multihop_fwd_bf16: Y is NULL");
  const void* src = X;
  for (int p = 0; p < max_power; ++p) {
    CIGN_REQUIRE(Y[p] != src || plan == nullptr || plan->p.rows == 0, CIGN_ERR_INVALID_ARGUMENT,
                 "multihop_fwd_bf16: Y[%d] aliases its input", p);
    const int rc = cign_spmm_bf16(plan, 0, src, F, Y[p], 1, ws, ws_bytes, stream);
    if (rc) return rc;
    src = Y[p];
  }
  return CIGN_OK;
}

size_t cign_multihop_workspace_bytes(const cign_spmm_plan* plan, int max_power, int64_t F) {
  if (plan == nullptr || F <= 0) return 0;
  const size_t state = max_power >= 2
                           ? (static_cast<size_t>(plan->p.rows) * F * sizeof(float) + 255) / 256 * 256
                           : 0;
  return state + partial_bytes(plan, F);
}

int cign_multihop_fwd(const cign_spmm_plan* plan, int max_power, const float* X, int64_t F,
                      float* const* Y, void* ws, size_t ws_bytes, cign_stream_t stream) {
  CIGN_REQUIRE(max_power >= 1, CIGN_ERR_INVALID_ARGUMENT,
               "multihop_fwd: max_power must be >= 1");
  CIGN_REQUIRE(Y != nullptr, CIGN_ERR_NULL_POINTER, "multihop_fwd: Y is NULL");
  int rc = check_dense(plan, X, F, Y[0], "multihop_fwd");
  if (rc) return rc;
  for (int p = 0; p < max_power; ++p) {
    CIGN_REQUIRE(Y[p] != nullptr || plan->p.rows == 0, CIGN_ERR_NULL_POINTER,
                 "multihop_fwd: Y[%d] is NULL", p);
    CIGN_REQUIRE(Y[p] != X || plan->p.rows == 0, CIGN_ERR_INVALID_ARGUMENT,
                 "multihop_fwd: Y[%d] aliases X", p);
    if (p > 0)
      CIGN_REQUIRE(Y[p] != Y[p - 1] || plan->p.rows == 0, CIGN_ERR_INVALID_ARGUMENT,
                   "multihop_fwd: Y[%d] aliases Y[%d]", p, p - 1);
  }
  const size_t need = partial_bytes(plan, F);
  CIGN_REQUIRE(ws_bytes >= need && (need == 0 || ws != nullptr), CIGN_ERR_INVALID_ARGUMENT,
               "multihop_fwd: workspace too small (%zu < %zu bytes)", ws_bytes, need);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* partial = static_cast<float*>(ws);
  const float* src = X;
  for (int p = 0; p < max_power; ++p) {
    rc = run_spmm(plan, 0, src, F, nullptr, Y[p], partial, s);
    if (rc) return rc;
    src = Y[p];
  }
  return CIGN_OK;
}

int cign_multihop_fwd_split(const cign_spmm_plan* plan, int max_power, const float* X0,
                            const float* X1, int64_t d, float* const* Y, void* ws,
                            size_t ws_bytes, cign_stream_t stream) {
  CIGN_REQUIRE(max_power >= 1, CIGN_ERR_INVALID_ARGUMENT,
               "multihop_fwd_split: max_power must be >= 1");
  CIGN_REQUIRE(Y != nullptr && X1 != nullptr, CIGN_ERR_NULL_POINTER,
               "multihop_fwd_split: NULL argument");
  const int64_t F = 2 * d;
  int rc = check_dense(plan, X0, F, Y[0], "multihop_fwd_split");
  if (rc) return rc;
  // the 256-float tiles of the float4 path for rows wider than 256 floats
  CIGN_REQUIRE(d % 256 == 0, CIGN_ERR_UNSUPPORTED,
               "multihop_fwd_split: d must be a multiple of 256 (got %lld)",
               static_cast<long long>(d));
  for (int p = 0; p < max_power; ++p) {
    CIGN_REQUIRE(Y[p] != nullptr || plan->p.rows == 0, CIGN_ERR_NULL_POINTER,
                 "multihop_fwd_split: Y[%d] is NULL", p);
    CIGN_REQUIRE(plan->p.rows == 0 || aligned16(Y[p]), CIGN_ERR_ALIGNMENT,
                 "multihop_fwd_split: Y[%d] must be 16-byte aligned", p);
  }
  CIGN_REQUIRE(plan->p.rows == 0 || (aligned16(X0) && aligned16(X1)), CIGN_ERR_ALIGNMENT,
               "multihop_fwd_split: X0 and X1 must be 16-byte aligned");
  const size_t need = partial_bytes(plan, F);
  CIGN_REQUIRE(ws_bytes >= need && (need == 0 || ws != nullptr), CIGN_ERR_INVALID_ARGUMENT,
               "multihop_fwd_split: workspace too small (%zu < %zu bytes)", ws_bytes, need);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* partial = static_cast<float*>(ws);
  CIGN_REQUIRE(partial == nullptr || aligned16(partial), CIGN_ERR_ALIGNMENT,
               "multihop_fwd_split: workspace must be 16-byte aligned");
  rc = launch_spmm_cfg<4, 2, 32>(plan->p, plan->seg_p, X0, F, nullptr, Y[0], partial, s, X1, d);
  if (rc) return rc;
  for (int p = 1; p < max_power; ++p) {
    rc = run_spmm(plan, 0, Y[p - 1], F, nullptr, Y[p], partial, s);
    if (rc) return rc;
  }
  return CIGN_OK;
}

int cign_multihop_bwd(const cign_spmm_plan* plan, int max_power, const float* const* G,
                      int64_t F, float* GX, void* ws, size_t ws_bytes, cign_stream_t stream) {
  CIGN_REQUIRE(max_power >= 1, CIGN_ERR_INVALID_ARGUMENT,
               "multihop_bwd: max_power must be >= 1");
  CIGN_REQUIRE(G != nullptr, CIGN_ERR_NULL_POINTER, "multihop_bwd: G is NULL");
  int rc = check_dense(plan, GX, F, GX, "multihop_bwd");
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int top = 0;  // highest power (1-based) with a gradient
  for (int p = max_power; p >= 1; --p)
    if (G[p - 1] != nullptr) { top = p; break; }
  const size_t bytes = static_cast<size_t>(plan->p.rows) * F * sizeof(float);
  if (top == 0) {
    if (bytes) CIGN_CHECK_CUDA(cudaMemsetAsync(GX, 0, bytes, s), "multihop_bwd: memset");
    return CIGN_OK;
  }
  const size_t need = cign_multihop_workspace_bytes(plan, max_power, F);
  CIGN_REQUIRE(ws_bytes >= need && (need == 0 || ws != nullptr), CIGN_ERR_INVALID_ARGUMENT,
               "multihop_bwd: workspace too small (%zu < %zu bytes)", ws_bytes, need);
  CIGN_REQUIRE(aligned16(ws), CIGN_ERR_ALIGNMENT, "multihop_bwd: ws must be 16-byte aligned");
  // workspace = [state buffer [rows, F] (max_power >= 2) | segment partials]
  const size_t state_bytes = max_power >= 2 ? (bytes + 255) / 256 * 256 : 0;
  float* state = static_cast<float*>(ws);
  float* partial = reinterpret_cast<float*>(static_cast<char*>(ws) + state_bytes);
  for (int p = 0; p < max_power; ++p)
    CIGN_REQUIRE(G[p] == nullptr || (G[p] != GX && G[p] != state) || plan->p.rows == 0,
                 CIGN_ERR_INVALID_ARGUMENT, "multihop_bwd: G[%d] aliases GX/ws", p);
  // u_top = G[top-1];  u_p = P^T u_{p+1} + G[p-1]  (p = top-1 .. 1);
  // GX = P^T u_1.  u_p lives in the state buffer for odd p and in GX for
  // even p, so the final SpMM reads the state buffer and writes GX.
  const float* u = G[top - 1];
  for (int p = top - 1; p >= 1; --p) {
    float* dst = (p & 1) ? state : GX;
    rc = run_spmm(plan, 1, u, F, G[p - 1], dst, partial, s);
    if (rc) return rc;
    u = dst;
  }
  return run_spmm(plan, 1, u, F, nullptr, GX, partial, s);
}

}  // extern "C"
