"""The net's dual input projection (generic_engine/model_cign.py:1162-1170):

    H = SiLU(x W0^T + b0) + eta * SiLU(x W1^T + b1)

as one autograd node: both projections in one GEMM (the stacked weight
[W0; W1] against x, so x is read once), then cign_silu_mix_fwd; the
backward forms [dz0 | dz1] and the eta gradient in one pass
(cign_silu_mix_bwd), then one weight-gradient GEMM and one fixed-order bias
column sum for both projections.  The same values as the reference's
expression up to the GEMMs' summation order (TF32 rules of the caller's
torch.backends settings apply to them)."""
from __future__ import annotations

import torch

from . import _lib
from .linear import _weight_grad, colsum


def silu_mix_forward(z: torch.Tensor, eta: torch.Tensor) -> torch.Tensor:
    """SiLU(z[:, :d]) + eta * SiLU(z[:, d:]) for z [n, 2d] (cign_silu_mix_fwd)."""
    lib = _lib.load_library()
    n, d2 = (int(s) for s in z.shape)
    out = torch.empty((n, d2 // 2), dtype=torch.float32, device=z.device)
    with _lib.DeviceGuard(z.device):
        rc = lib.cign_silu_mix_fwd(n, d2 // 2, _lib.ptr(z), _lib.ptr(eta), _lib.ptr(out),
                                   _lib.stream_of(z))
    _lib.check(rc, "cign_silu_mix_fwd")
    return out


def silu_mix_backward(g: torch.Tensor, z: torch.Tensor, eta: torch.Tensor):
    """(grad_z [n, 2d], grad_eta []) of silu_mix_forward (cign_silu_mix_bwd)."""
    lib = _lib.load_library()
    n, d2 = (int(s) for s in z.shape)
    gz = torch.empty_like(z)
    geta = torch.empty((), dtype=torch.float32, device=z.device)
    ws = _lib.workspace(lib.cign_silu_mix_bwd_workspace_bytes(n, d2 // 2), z.device)
    with _lib.DeviceGuard(z.device):
        rc = lib.cign_silu_mix_bwd(n, d2 // 2, _lib.ptr(g), _lib.ptr(z), _lib.ptr(eta),
                                   _lib.ptr(gz), _lib.ptr(geta), _lib.ptr(ws), ws.numel(),
                                   _lib.stream_of(z))
    _lib.check(rc, "cign_silu_mix_bwd")
    return gz, geta


class _DualInputProjectionFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w0, b0, w1, b1, eta):
        x = x.contiguous()
        d = int(w0.size(0))
        z = torch.addmm(torch.cat([b0, b1]), x, torch.cat([w0, w1]).t())     # [n, 2d]
        ctx.save_for_backward(x, z, eta)
        ctx.d = d
        return silu_mix_forward(z, eta.reshape(1))

    @staticmethod
    def backward(ctx, g):
        x, z, eta = ctx.saved_tensors
        d = ctx.d
        gz, geta = silu_mix_backward(g.contiguous(), z, eta.reshape(1))
        gw = _weight_grad(gz, x)                                               # [2d, in]
        gb = colsum(gz)                                                        # [2d]
        return (None, gw[:d], gb[:d], gw[d:], gb[d:], geta.reshape(eta.shape))


def dual_input_projection(x: torch.Tensor, w0: torch.Tensor, b0: torch.Tensor, w1: torch.Tensor,
                          b1: torch.Tensor, eta: torch.Tensor) -> torch.Tensor:
    """SiLU(x w0^T + b0) + eta * SiLU(x w1^T + b1) for a 2-D CUDA float32 x
    (x gets no gradient: it is the net's input)."""
    if x.requires_grad:
        raise ValueError("dual_input_projection: x must not require a gradient")
    return _DualInputProjectionFn.apply(x, w0, b0, w1, b1, eta)
