"""Shared autograd Function of the Clifford pack family (cign_pack_fwd/bwd).

Modes (numbers as in include/cign_sm100.h):
  interaction 0 = "old": D = SiLU(H*T_C), W = H*T_C - C*T_H
  interaction 1 = "new": D = SiLU((H*T_C + C*T_H)/2), W = o((H*T_C - C*T_H)/2)
  outer       0 = none, 1 = tanh (o above)
  weighting   0 = "old": out = cat_k a_k [W_k, D_k]          -> [N, 2KD]
  weighting   1 = "new": out = [sum_k a_k D_k, sum_k a_k W_k] -> [N, 2D]
"""
from __future__ import annotations

from typing import Optional, Sequence

import torch

from . import _lib


def pack_forward(H, C, props: Sequence[torch.Tensor], alpha: Optional[torch.Tensor],
                 interaction: int, outer: int, weighting: int) -> torch.Tensor:
    lib = _lib.load_library()
    n, D = (int(s) for s in H.shape)
    K = len(props)
    out_cols = 2 * K * D if weighting == 0 else 2 * D
    out = torch.empty((n, out_cols), dtype=torch.float32, device=H.device)
    arr = _lib.ptr_array(props)
    with _lib.DeviceGuard(H.device):
        rc = lib.cign_pack_fwd(n, D, K, int(interaction), int(outer), int(weighting), _lib.ptr(H),
                               _lib.ptr(C), arr, 2 * D, _lib.ptr(alpha), _lib.ptr(out),
                               _lib.stream_of(H))
    _lib.check(rc, "cign_pack_fwd")
    return out


def gate_pack_supported(H, C, props: Sequence[torch.Tensor]) -> bool:
    """Whether cign_gate_pack_fwd (hop gate inside the pack forward) takes
    these operands: D % 4 == 0, D <= 1024, 1 <= K <= 8, 16-byte aligned."""
    D, K = int(H.size(1)), len(props)
    return (D % 4 == 0 and D <= 1024 and 1 <= K <= 8
            and all(t.data_ptr() % 16 == 0 for t in (H, C, *props)))


def gate_pack_forward(H, C, props: Sequence[torch.Tensor], gate_w, gate_b, gate_mode: int,
                      interaction: int, outer: int, weighting: int):
    """(G, alpha): the hop gate's alpha [N, K] and the pack that uses it, in
    one pass over H and C (cign_gate_pack_fwd)."""
    lib = _lib.load_library()
    n, D = (int(s) for s in H.shape)
    K = len(props)
    out_cols = 2 * K * D if weighting == 0 else 2 * D
    out = torch.empty((n, out_cols), dtype=torch.float32, device=H.device)
    alpha = torch.empty((n, K), dtype=torch.float32, device=H.device)
    with _lib.DeviceGuard(H.device):
        rc = lib.cign_gate_pack_fwd(n, D, K, int(gate_mode), int(interaction), int(outer),
                                    int(weighting), _lib.ptr(H), _lib.ptr(C),
                                    _lib.ptr_array(props), 2 * D, _lib.ptr(gate_w.contiguous()),
                                    _lib.ptr(gate_b.contiguous()), _lib.ptr(alpha),
                                    _lib.ptr(out), _lib.stream_of(H))
    _lib.check(rc, "cign_gate_pack_fwd")
    return out, alpha


def pack_proj_supported(D: int, K: int, dout: int) -> bool:
    """Shapes the tcgen05 pack + proj GEMM (cign_pack_proj_gemm_tf32) takes."""
    return D % 32 == 0 and 1 <= K <= 8 and dout % 32 == 0 and 32 <= dout <= 512


def pack_proj_call(H, C, props: Sequence[torch.Tensor], alpha: torch.Tensor,
                   weight: torch.Tensor, bias: torch.Tensor, keep_g: bool):
    """(out, G or None, workspace) of one cign_pack_proj_gemm_tf32 call; the
    workspace holds the device status word that pack_proj_status reads."""
    lib = _lib.load_library()
    n, D = (int(s) for s in H.shape)
    K = len(props)
    dout = int(weight.size(0))
    weight = weight.contiguous()
    out = torch.empty((n, dout), dtype=torch.float32, device=H.device)
    G = torch.empty((n, 2 * K * D), dtype=torch.float32, device=H.device) if keep_g else None
    ws = _lib.workspace(lib.cign_pack_proj_workspace_bytes(D, K, dout), H.device)
    with _lib.DeviceGuard(H.device):
        rc = lib.cign_pack_proj_gemm_tf32(n, D, K, dout, _lib.ptr(H), _lib.ptr(C),
                                          _lib.ptr_array(props), 2 * D, _lib.ptr(alpha),
                                          _lib.ptr(weight), _lib.ptr(bias.contiguous()),
                                          _lib.ptr(out), _lib.ptr(G), _lib.ptr(ws), ws.numel(),
                                          _lib.stream_of(H))
    _lib.check(rc, "cign_pack_proj_gemm_tf32")
    return out, G, ws


def pack_proj_forward(H, C, props: Sequence[torch.Tensor], alpha: torch.Tensor,
                      weight: torch.Tensor, bias: torch.Tensor, keep_g: bool):
    """(G @ weight.T + bias, G or None) for G = pack(H, C, props, alpha) with the
    production switches (interaction "new", outer none, weighting "old"),
    G never stored unless keep_g; TF32 tensor-core products, fp32 sums."""
    out, G, _ = pack_proj_call(H, C, props, alpha, weight, bias, keep_g)
    return out, G


def pack_proj_status(ws: torch.Tensor, D: int, K: int, dout: int) -> None:
    """Raise if a bounded device-side wait of the call that used `ws` expired
    (synchronises the current stream)."""
    lib = _lib.load_library()
    with _lib.DeviceGuard(ws.device):
        rc = lib.cign_pack_proj_status(_lib.ptr(ws), int(D), int(K), int(dout),
                                       _lib.stream_of(ws))
    _lib.check(rc, "cign_pack_proj_status")


def pack_backward(grad_out, H, C, props, alpha, interaction, outer, weighting, need_alpha: bool):
    lib = _lib.load_library()
    n, D = (int(s) for s in H.shape)
    K = len(props)
    gH = torch.empty_like(H)
    gC = torch.empty_like(C)
    gP = [torch.empty_like(p) for p in props]
    gA = torch.empty((n, K), dtype=torch.float32, device=H.device) if need_alpha else None
    with _lib.DeviceGuard(H.device):
        rc = lib.cign_pack_bwd(n, D, K, int(interaction), int(outer), int(weighting),
                               _lib.ptr(grad_out), _lib.ptr(H), _lib.ptr(C), _lib.ptr_array(props),
                               2 * D, _lib.ptr(alpha), _lib.ptr(gH), _lib.ptr(gC),
                               _lib.ptr_array(gP), 2 * D, 0, _lib.ptr(gA), _lib.stream_of(H))
    _lib.check(rc, "cign_pack_bwd")
    return gH, gC, gP, gA


class PackFunction(torch.autograd.Function):
    """apply(interaction, outer, weighting, H, C, alpha_or_None, *props)."""

    @staticmethod
    def forward(ctx, interaction, outer, weighting, H, C, alpha, *props):
        props = [p.to(torch.float32).contiguous() for p in props]
        out = pack_forward(H, C, props, alpha, interaction, outer, weighting)
        ctx.modes = (int(interaction), int(outer), int(weighting))
        ctx.has_alpha = alpha is not None
        ctx.save_for_backward(H, C, *( [alpha] if alpha is not None else [] ), *props)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        saved = ctx.saved_tensors
        H, C = saved[0], saved[1]
        if ctx.has_alpha:
            alpha, props = saved[2], list(saved[3:])
        else:
            alpha, props = None, list(saved[2:])
        need_alpha = ctx.has_alpha and ctx.needs_input_grad[5]
        gH, gC, gP, gA = pack_backward(grad_out.to(torch.float32).contiguous(), H, C, props, alpha,
                                       *ctx.modes, need_alpha=need_alpha)
        return (None, None, None, gH, gC, gA, *gP)


def normalize_alpha(alpha, N: int, K: int) -> Optional[torch.Tensor]:
    """None stays None (all-ones weights, no gradient); [N,K,1] -> [N,K]
    (fused_clifford_pack.py:210-217)."""
    if alpha is None:
        return None
    if alpha.dim() == 3 and alpha.size(-1) == 1:
        alpha = alpha.squeeze(-1)
    if tuple(alpha.shape) != (N, K):
        raise ValueError(f"Expected alpha {(N, K)}, got {tuple(alpha.shape)}")
    return alpha.to(dtype=torch.float32).contiguous()


def check_inputs(H_norm, C_norm, propagated):
    if H_norm.dim() != 2 or C_norm.shape != H_norm.shape:
        raise ValueError("H_norm and C_norm must both be [N,D]")
    N, D = H_norm.shape
    if len(propagated) <= 0:
        raise ValueError("propagated cannot be empty")
    for p in propagated:
        if tuple(p.shape) != (N, 2 * D):
            raise ValueError(f"Every propagated tensor must be {(N, 2 * D)}, got {tuple(p.shape)}")
    if not H_norm.is_cuda:
        raise RuntimeError("Clifford pack requires CUDA tensors (no CPU fallback).")
    return int(N), int(D)


def run_pack(H_norm, C_norm, propagated, alpha, interaction, outer, weighting):
    N, D = check_inputs(H_norm, C_norm, propagated)
    K = len(propagated)
    H = H_norm.to(dtype=torch.float32).contiguous()
    C = C_norm.to(dtype=torch.float32).contiguous()
    A = normalize_alpha(alpha, N, K)
    return PackFunction.apply(int(interaction), int(outer), int(weighting), H, C, A, *propagated)
