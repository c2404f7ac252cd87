// Per-channel Clifford interaction of the pack kernels (pack.cu) and of the
// pack-prologue GEMM (pack_proj.cu), so both evaluate the same expressions.
#pragma once

#include "common.cuh"

namespace cign {

// D/W of one channel and their partial derivatives w.r.t. b_hr and b_rh
// (the reference's compute_dw, switch pack cu:22-58, plus the "old"
// interaction of fused_clifford_pack_cuda.cu:47-49).
struct DW {
  float D, W, dD_hr, dD_rh, dW_hr, dW_rh;
};
__device__ __forceinline__ DW interact(float bhr, float brh, int interaction, int outer) {
  DW r;
  if (interaction == 0) {
    r.D = silu_f(bhr);
    r.W = bhr - brh;
    r.dD_hr = silu_grad_f(bhr);
    r.dD_rh = 0.0f;
    r.dW_hr = 1.0f;
    r.dW_rh = -1.0f;
  } else {
    const float sym = 0.5f * (bhr + brh);
    const float anti = 0.5f * (bhr - brh);
    r.D = silu_f(sym);
    const float sd = 0.5f * silu_grad_f(sym);
    r.dD_hr = sd;
    r.dD_rh = sd;
    float dw;
    if (outer == 1) {
      r.W = tanhf(anti);
      dw = 1.0f - r.W * r.W;
    } else {
      r.W = anti;
      dw = 1.0f;
    }
    r.dW_hr = 0.5f * dw;
    r.dW_rh = -0.5f * dw;
  }
  return r;
}
// Forward-only variant (no derivatives).
__device__ __forceinline__ void interact_fwd(float bhr, float brh, int interaction, int outer,
                                             float& D, float& W) {
  if (interaction == 0) {
    D = silu_f(bhr);
    W = bhr - brh;
  } else {
    D = silu_f(0.5f * (bhr + brh));
    const float anti = 0.5f * (bhr - brh);
    W = outer == 1 ? tanhf(anti) : anti;
  }
}

}  // namespace cign
