"""The model's output LayerNorm over the concatenated block states,
LayerNorm(torch.cat(states, -1)) of GraphCliffordNet
(generic_engine/model_cign.py:1195-1201), computed by cign_jk_ln_fwd/bwd
straight from the state tensors: no concatenated copy forward, no split of
the gradient backward, and the LayerNorm weight/bias gradients summed in a
fixed order.  Same values as torch.nn.functional.layer_norm up to fp32
rounding of the mean/variance."""
from __future__ import annotations

from typing import Sequence

import torch

from . import _lib


def jk_norm_supported(states: Sequence[torch.Tensor]) -> bool:
    if not states or not all(s.is_cuda and s.dtype == torch.float32 and s.dim() == 2
                             for s in states):
        return False
    w = states[0].size(1)
    n = states[0].size(0)
    return (all(s.shape == (n, w) for s in states) and w % 4 == 0
            and len(states) * w <= 2048 and len(states) <= 8)


class _JKLayerNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, weight, bias, eps, *states):
        lib = _lib.load_library()
        states = [s.contiguous() for s in states]
        n, W = (int(v) for v in states[0].shape)
        S = len(states)
        dev = states[0].device
        y = torch.empty((n, S * W), dtype=torch.float32, device=dev)
        mean = torch.empty((n,), dtype=torch.float32, device=dev)
        rstd = torch.empty((n,), dtype=torch.float32, device=dev)
        with _lib.DeviceGuard(dev):
            rc = lib.cign_jk_ln_fwd(n, S, W, _lib.ptr_array(states), _lib.ptr(weight),
                                    _lib.ptr(bias), float(eps), _lib.ptr(y), _lib.ptr(mean),
                                    _lib.ptr(rstd), _lib.stream_of(y))
        _lib.check(rc, "cign_jk_ln_fwd")
        ctx.save_for_backward(weight, mean, rstd, *states)
        return y

    @staticmethod
    def backward(ctx, gy):
        lib = _lib.load_library()
        weight, mean, rstd, *states = ctx.saved_tensors
        gy = gy.contiguous()
        n, W = (int(v) for v in states[0].shape)
        S = len(states)
        dev = gy.device
        gs = [torch.empty_like(s) for s in states]
        gw = torch.empty_like(weight)
        gb = torch.empty_like(weight)
        ws = _lib.workspace(lib.cign_jk_ln_workspace_bytes(n, S * W), dev)
        with _lib.DeviceGuard(dev):
            rc = lib.cign_jk_ln_bwd(n, S, W, _lib.ptr(gy), _lib.ptr_array(states),
                                    _lib.ptr(weight), _lib.ptr(mean), _lib.ptr(rstd),
                                    _lib.ptr_array(gs), _lib.ptr(gw), _lib.ptr(gb),
                                    _lib.ptr(ws), ws.numel(), _lib.stream_of(gy))
        _lib.check(rc, "cign_jk_ln_bwd")
        return (gw, gb, None, *gs)


def jk_layer_norm(states: Sequence[torch.Tensor], weight: torch.Tensor, bias: torch.Tensor,
                  eps: float) -> torch.Tensor:
    """LayerNorm(torch.cat(states, -1), weight, bias, eps) for equal-width
    CUDA fp32 states (row width at most 2048 floats in total)."""
    if not jk_norm_supported(states):
        raise ValueError("jk_layer_norm needs 1..8 CUDA fp32 [N, W] states, W % 4 == 0, "
                         "len(states) * W <= 2048")
    if weight.numel() != len(states) * states[0].size(1):
        raise ValueError("weight/bias must cover the concatenated width")
    return _JKLayerNormFn.apply(weight.contiguous(), bias.contiguous(), float(eps), *states)
