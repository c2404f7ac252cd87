// The net's dual input projection after its GEMM
// (generic_engine/model_cign.py:1162-1170):
//   H = SiLU(x W0^T + b0) + eta * SiLU(x W1^T + b1)
// with both projections computed by one GEMM into z = [z0 | z1] ([n, 2d]).
// Forward: out = silu(z0) + eta * silu(z1), the product and the sum rounded
// separately (as torch's mul and add kernels).  Backward: grad_z0 = g *
// silu'(z0), grad_z1 = (eta * g) * silu'(z1), grad_eta = sum of g * silu(z1)
// over all elements -- per block over a fixed row range in a fixed order,
// then over the blocks by the fixed-order column sum.
#include <algorithm>
#include <initializer_list>

#include "common.cuh"

namespace cign {
namespace {

constexpr int kMixThreads = 256;
constexpr int kMixWarps = kMixThreads / 32;
constexpr int64_t kMixRows = 32;  // rows per backward block (fixed: the eta sum's order)

// One warp per row, lanes over the row's float4 columns.
__global__ void __launch_bounds__(kMixThreads)
silu_mix_fwd_kernel(int64_t n, int64_t d, const float* __restrict__ z,
                    const float* __restrict__ eta_p, float* __restrict__ out) {
  const float eta = __ldg(eta_p);
  const int lane = threadIdx.x & 31;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * kMixWarps + (threadIdx.x >> 5); r < n;
       r += static_cast<int64_t>(gridDim.x) * kMixWarps) {
    const float* za = z + r * 2 * d;
    for (int64_t c = static_cast<int64_t>(lane) * 4; c < d; c += 128) {
      const float4 a = ldg_vec<4>(za + c);
      const float4 b = ldg_vec<4>(za + d + c);
      float4 o;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        vel(o, j) = __fadd_rn(silu_f(vel(a, j)), __fmul_rn(eta, silu_f(vel(b, j))));
      st_vec(out + r * d + c, o);
    }
  }
}

// Block b covers rows [b * kMixRows, (b + 1) * kMixRows), warp w its rows
// w, w + kMixWarps, ...; each lane sums its g * silu(z1) terms in row order.
__global__ void __launch_bounds__(kMixThreads)
silu_mix_bwd_kernel(int64_t n, int64_t d, const float* __restrict__ g,
                    const float* __restrict__ z, const float* __restrict__ eta_p,
                    float* __restrict__ gz, float* __restrict__ part) {
  __shared__ float red[kMixWarps];
  const float eta = __ldg(eta_p);
  const int lane = threadIdx.x & 31;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kMixRows;
  const int64_t r1 = r0 + kMixRows < n ? r0 + kMixRows : n;
  float acc = 0.0f;
  for (int64_t r = r0 + (threadIdx.x >> 5); r < r1; r += kMixWarps) {
    const float* za = z + r * 2 * d;
    float* ga_row = gz + r * 2 * d;
    for (int64_t c = static_cast<int64_t>(lane) * 4; c < d; c += 128) {
      const float4 gv = ldg_vec<4>(g + r * d + c);
      const float4 a = ldg_vec<4>(za + c);
      const float4 b = ldg_vec<4>(za + d + c);
      float4 ga, gb;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        vel(ga, j) = __fmul_rn(vel(gv, j), silu_grad_f(vel(a, j)));
        vel(gb, j) = __fmul_rn(__fmul_rn(eta, vel(gv, j)), silu_grad_f(vel(b, j)));
        acc = __fadd_rn(acc, __fmul_rn(vel(gv, j), silu_f(vel(b, j))));
      }
      st_vec(ga_row + c, ga);
      st_vec(ga_row + d + c, gb);
    }
  }
  acc = warp_sum(acc);
  if (lane == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = red[0];
    for (int w = 1; w < kMixWarps; ++w) t += red[w];
    part[blockIdx.x] = t;
  }
}

int64_t mix_blocks(int64_t n) { return (n + kMixRows - 1) / kMixRows; }

int check_mix(int64_t n, int64_t d, std::initializer_list<const void*> ptrs, const char* name) {
  CIGN_REQUIRE(n >= 0 && d >= 4 && d % 4 == 0, CIGN_ERR_UNSUPPORTED,
               "%s: needs d %% 4 == 0 (got n=%lld, d=%lld)", name, static_cast<long long>(n),
               static_cast<long long>(d));
  if (n == 0) return CIGN_OK;
  for (const void* p : ptrs) {
    CIGN_REQUIRE(p != nullptr, CIGN_ERR_NULL_POINTER, "%s: NULL argument", name);
    CIGN_REQUIRE(aligned16(p), CIGN_ERR_ALIGNMENT, "%s: tensors must be 16-byte aligned", name);
  }
  return CIGN_OK;
}

}  // namespace
}  // namespace cign

using namespace cign;

extern "C" {

int cign_silu_mix_fwd(int64_t n, int64_t d, const float* z, const float* eta, float* out,
                      cign_stream_t stream) {
  int rc = check_mix(n, d, {z, out}, "silu_mix_fwd");
  if (rc) return rc;
  if (n == 0) return CIGN_OK;
  CIGN_REQUIRE(eta != nullptr, CIGN_ERR_NULL_POINTER, "silu_mix_fwd: NULL eta");
  const int64_t blocks = std::min<int64_t>((n + kMixWarps - 1) / kMixWarps, 148 * 16);
  silu_mix_fwd_kernel<<<static_cast<unsigned>(blocks), kMixThreads, 0,
                        static_cast<cudaStream_t>(stream)>>>(n, d, z, eta, out);
  CIGN_CHECK_LAUNCH("silu_mix_fwd_kernel");
  return CIGN_OK;
}

size_t cign_silu_mix_bwd_workspace_bytes(int64_t n, int64_t d) {
  if (n <= 0 || d <= 0) return 0;
  return static_cast<size_t>(mix_blocks(n)) * sizeof(float);
}

int cign_silu_mix_bwd(int64_t n, int64_t d, const float* grad_out, const float* z,
                      const float* eta, float* grad_z, float* grad_eta, void* ws,
                      size_t ws_bytes, cign_stream_t stream) {
  int rc = check_mix(n, d, {grad_out, z, grad_z}, "silu_mix_bwd");
  if (rc) return rc;
  CIGN_REQUIRE(eta != nullptr && grad_eta != nullptr, CIGN_ERR_NULL_POINTER,
               "silu_mix_bwd: NULL eta / grad_eta");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n == 0) {
    CIGN_CHECK_CUDA(cudaMemsetAsync(grad_eta, 0, sizeof(float), s), "silu_mix_bwd: memset");
    return CIGN_OK;
  }
  CIGN_REQUIRE(ws != nullptr && ws_bytes >= cign_silu_mix_bwd_workspace_bytes(n, d),
               CIGN_ERR_INVALID_ARGUMENT, "silu_mix_bwd: workspace too small");
  const int64_t blocks = mix_blocks(n);
  CIGN_REQUIRE(blocks < (1ll << 31), CIGN_ERR_UNSUPPORTED, "silu_mix_bwd: too large");
  float* part = static_cast<float*>(ws);
  silu_mix_bwd_kernel<<<static_cast<unsigned>(blocks), kMixThreads, 0, s>>>(n, d, grad_out, z,
                                                                            eta, grad_z, part);
  CIGN_CHECK_LAUNCH("silu_mix_bwd_kernel");
  return colsum_rows(part, grad_eta, nullptr, nullptr, blocks, 1, 1, s);
}

}  // extern "C"
