"""Fused hop gate of the CIGN block (generic_engine/model_cign.py:721-749).

``fused_hop_gate(H_norm, C_norm, weight, bias, score_mode)`` returns
``softmax(gate_input @ weight.T + bias, -1)`` as [N, K] with
``gate_input = [H + C | |H - C|]`` (score mode "new") or ``[H | C]`` ("old"),
computed by cign_hop_gate_fwd/_bwd without materialising the gate input;
gradients flow to H_norm, C_norm, weight and bias.
"""
from __future__ import annotations

import torch

from . import _lib

MAX_HOPS = 8


def hop_gate_forward_raw(h, c, weight, bias, mode: int) -> torch.Tensor:
    """alpha [N, K] (cign_hop_gate_fwd)."""
    lib = _lib.load_library()
    n, d = h.shape
    k = int(weight.size(0))
    alpha = torch.empty((n, k), dtype=torch.float32, device=h.device)
    with _lib.DeviceGuard(h.device):
        rc = lib.cign_hop_gate_fwd(n, d, k, int(mode), _lib.ptr(h), _lib.ptr(c), _lib.ptr(weight),
                                   _lib.ptr(bias), _lib.ptr(alpha), _lib.stream_of(h))
    _lib.check(rc, "cign_hop_gate_fwd")
    return alpha


def hop_gate_backward_raw(h, c, weight, alpha, grad_alpha, mode: int, grad_h, grad_c,
                          accumulate: bool = False, add_h=None, add_c=None, add_ld: int = 0):
    """Writes grad_h/grad_c (see cign_hop_gate_bwd); returns (grad_w, grad_b)."""
    lib = _lib.load_library()
    n, d = h.shape
    k = int(weight.size(0))
    gw = torch.empty_like(weight)
    gb = torch.empty((k,), dtype=torch.float32, device=h.device)
    ws = _lib.workspace(lib.cign_hop_gate_bwd_workspace_bytes(n, d, k), h.device)
    with _lib.DeviceGuard(h.device):
        rc = lib.cign_hop_gate_bwd(n, d, k, int(mode), _lib.ptr(h), _lib.ptr(c), _lib.ptr(weight),
                                   _lib.ptr(alpha), _lib.ptr(grad_alpha.contiguous()),
                                   _lib.ptr(grad_h), _lib.ptr(grad_c), _lib.ptr(gw), _lib.ptr(gb),
                                   1 if accumulate else 0, add_h, add_c, int(add_ld),
                                   _lib.ptr(ws), ws.numel(), _lib.stream_of(h))
    _lib.check(rc, "cign_hop_gate_bwd")
    return gw, gb


class _HopGateFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, c, weight, bias, mode):
        lib = _lib.load_library()
        n, d = h.shape
        k = int(weight.size(0))
        alpha = torch.empty((n, k), dtype=torch.float32, device=h.device)
        with _lib.DeviceGuard(h.device):
            rc = lib.cign_hop_gate_fwd(n, d, k, int(mode), _lib.ptr(h), _lib.ptr(c),
                                       _lib.ptr(weight), _lib.ptr(bias), _lib.ptr(alpha),
                                       _lib.stream_of(h))
        _lib.check(rc, "cign_hop_gate_fwd")
        ctx.save_for_backward(h, c, weight, alpha)
        ctx.mode = int(mode)
        return alpha

    @staticmethod
    def backward(ctx, grad_alpha):
        h, c, weight, alpha = ctx.saved_tensors
        lib = _lib.load_library()
        n, d = h.shape
        k = int(weight.size(0))
        gh = torch.empty_like(h)
        gc = torch.empty_like(c)
        gw = torch.empty_like(weight)
        gb = torch.empty((k,), dtype=torch.float32, device=h.device)
        ws = _lib.workspace(lib.cign_hop_gate_bwd_workspace_bytes(n, d, k), h.device)
        with _lib.DeviceGuard(h.device):
            rc = lib.cign_hop_gate_bwd(n, d, k, ctx.mode, _lib.ptr(h), _lib.ptr(c),
                                       _lib.ptr(weight), _lib.ptr(alpha),
                                       _lib.ptr(grad_alpha.contiguous()), _lib.ptr(gh),
                                       _lib.ptr(gc), _lib.ptr(gw), _lib.ptr(gb), 0, None, None, 0,
                                       _lib.ptr(ws), ws.numel(), _lib.stream_of(h))
        _lib.check(rc, "cign_hop_gate_bwd")
        return gh, gc, gw, gb, None


def fused_hop_gate(H_norm: torch.Tensor, C_norm: torch.Tensor, weight: torch.Tensor,
                   bias: torch.Tensor, score_mode: str = "new") -> torch.Tensor:
    if score_mode not in ("new", "old"):
        raise ValueError(f"score_mode must be 'new' or 'old', got {score_mode!r}")
    if H_norm.shape != C_norm.shape or H_norm.dim() != 2:
        raise ValueError("H_norm and C_norm must be [N, D] of the same shape")
    k = int(weight.size(0))
    if not (1 <= k <= MAX_HOPS) or weight.shape != (k, 2 * H_norm.size(1)) or bias.shape != (k,):
        raise ValueError("weight must be [K, 2D] and bias [K], 1 <= K <= 8")
    for t in (H_norm, C_norm, weight, bias):
        if t.dtype != torch.float32 or t.device.type != "cuda":
            raise TypeError("fused_hop_gate requires CUDA float32 tensors")
    return _HopGateFn.apply(H_norm.contiguous(), C_norm.contiguous(), weight.contiguous(),
                            bias.contiguous(), 1 if score_mode == "new" else 0)
