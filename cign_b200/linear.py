"""Linear layer whose backward sums the bias gradient with the library's
fixed-order column sum (cign_colsum_f32) instead of autograd's
grad.sum(0), and splits the weight-gradient reduction over the rows into
a batched GEMM when the input is narrow (the [rows, 300] input projection,
whose one-piece GEMM leaves most SMs idle).  Same values as nn.Linear
(TF32 rules of the caller's torch.backends settings apply to the GEMMs)."""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib


def colsum(a: torch.Tensor) -> torch.Tensor:
    """Fixed-order column sums of a [n, c] CUDA float32 matrix."""
    a = a.contiguous()
    lib = _lib.load_library()
    n, c = (int(s) for s in a.shape)
    out = torch.empty((c,), dtype=torch.float32, device=a.device)
    ws = _lib.workspace(lib.cign_colsum_workspace_bytes(n, c), a.device)
    with _lib.DeviceGuard(a.device):
        rc = lib.cign_colsum_f32(n, c, _lib.ptr(a), _lib.ptr(out), _lib.ptr(ws), ws.numel(),
                                 _lib.stream_of(a))
    _lib.check(rc, "cign_colsum_f32")
    return out


_SPLIT_ROWS = 8192   # rows per weight-gradient slice for narrow inputs
_NARROW = 512        # inputs narrower than this get the split reduction


def _weight_grad(g: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    n = x.size(0)
    if x.size(1) >= _NARROW or n < 2 * _SPLIT_ROWS:
        return g.t().mm(x)
    s = n // _SPLIT_ROWS
    m = s * _SPLIT_ROWS
    part = torch.bmm(g[:m].view(s, _SPLIT_ROWS, -1).transpose(1, 2),
                     x[:m].view(s, _SPLIT_ROWS, -1)).sum(0)
    if m < n:
        part = part + g[m:].t().mm(x[m:])
    return part


class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias):
        x = x.contiguous()
        ctx.save_for_backward(x, weight)
        ctx.has_bias = bias is not None
        if bias is None:
            return x.mm(weight.t())
        return torch.addmm(bias, x, weight.t())

    @staticmethod
    def backward(ctx, g):
        x, weight = ctx.saved_tensors
        g = g.contiguous()
        gx = g.mm(weight) if ctx.needs_input_grad[0] else None
        gw = _weight_grad(g, x) if ctx.needs_input_grad[1] else None
        gb = colsum(g) if ctx.has_bias and ctx.needs_input_grad[2] else None
        return gx, gw, gb


def linear(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor]) -> torch.Tensor:
    """y = x @ weight.T + bias for a 2-D CUDA float32 x."""
    if not x.is_cuda or x.dim() != 2:
        return torch.nn.functional.linear(x, weight, bias)
    return _LinearFn.apply(x, weight, bias)
