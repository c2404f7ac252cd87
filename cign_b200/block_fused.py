"""The middle of a CIGN block as one autograd node:

    HC     = [H_norm | C_norm]
    T^p    = P^p HC,  p in order_set                 (k-hop propagation)
    alpha  = softmax(hop_gate([H+C, |H-C|]))         (hop gate)
    G_raw  = Clifford pack(H_norm, C_norm, T, alpha)
(the hop gate and the pack run as one kernel in the forward,
cign_gate_pack_fwd)

(generic_engine/model_cign.py:781-925, production switches: interaction
"new", outer nonlinearity "none", alpha weighting "old").  Run op by op,
autograd accumulates the gradients of H_norm and C_norm from four
consumers each with separate add kernels, several of them reading
non-contiguous slices of the [H_norm | C_norm] gradient.  Here the backward
runs pack -> k-hop propagation -> hop gate, and the hop-gate backward
kernel adds the pack's gradients and both halves of the propagation's
gradient into H_norm's and C_norm's gradients in the same pass.  The
forward values are those of the op-by-op composition.
"""
from __future__ import annotations

from typing import Sequence

import torch

from . import _lib, _pack
from .hop_gate import hop_gate_backward_raw, hop_gate_forward_raw
from .linear import _weight_grad, colsum
from .multihop_csr_pipeline import (GenericMultiHopCSRGraphOperator,
                                    HybridNative3TailCSRGraphOperator, MultiHopCSR3GraphOperator)
from .plans import SpmmPlan, spmm_plan_for

PACK_MODES = (1, 0, 0)  # interaction "new", outer none, weighting "old"
# pack + proj on the tcgen05 pack-prologue GEMM (TF32 matmuls allowed):
# None = when G_raw is not kept (large graphs: no G write at all, and many
# row tiles per SM); True/False = always/never.  When G_raw is kept, writing
# it from the GEMM costs more than the separate pack kernel's write.
USE_TCGEN05_PACK_PROJ = None


def native_spmm_plan(operator):
    """The propagator behind a k-hop operator: the SpmmPlan of a
    multihop_csr_pipeline operator, or the row-partitioned operator itself
    (cign_b200.distributed.DistMultiHop, which has the same forward(x, K) /
    backward(grads, F) pair); None for other operators."""
    if getattr(operator, "is_row_partitioned", False):
        return operator
    if isinstance(operator, MultiHopCSR3GraphOperator):
        return operator.plan.spmm
    if isinstance(operator, HybridNative3TailCSRGraphOperator):
        return operator.native3.plan.spmm
    if isinstance(operator, GenericMultiHopCSRGraphOperator):
        return spmm_plan_for(operator.base.csr, operator.base.csr_t)
    return None


class _PropagateGatePackFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, H, C, gate_w, gate_b, plan, order_set, gate_mode):
        H = H.contiguous()
        C = C.contiguous()
        D = H.size(1)
        props = _propagate(H, C, plan, order_set)
        G, alpha = _gate_pack(H, C, props, gate_w, gate_b, gate_mode)
        ctx.save_for_backward(H, C, gate_w, alpha, *props)
        ctx.plan, ctx.order_set, ctx.gate_mode, ctx.D = plan, tuple(order_set), gate_mode, D
        return G

    @staticmethod
    def backward(ctx, gG):
        H, C, gate_w, alpha, *props = ctx.saved_tensors
        gH, gC, gw, gb = _gate_pack_backward(ctx, gG, H, C, gate_w, alpha, props)
        return gH, gC, gw, gb, None, None, None


def _gate_pack(H, C, props, gate_w, gate_b, gate_mode):
    """(G, alpha): hop gate and pack in one pass over H and C where the shape
    allows, else the two kernels."""
    if _pack.gate_pack_supported(H, C, props):
        return _pack.gate_pack_forward(H, C, props, gate_w, gate_b, gate_mode, *PACK_MODES)
    alpha = hop_gate_forward_raw(H, C, gate_w, gate_b, gate_mode)
    return _pack.pack_forward(H, C, props, alpha, *PACK_MODES), alpha


def _propagate(H, C, plan, order_set):
    if (isinstance(plan, SpmmPlan) and H.size(1) % 256 == 0
            and H.data_ptr() % 16 == 0 and C.data_ptr() % 16 == 0):
        ys = plan.forward_split(H, C, max(order_set))  # no [H | C] copy
    else:
        ys = plan.forward(torch.cat([H, C], 1), max(order_set))
    return [ys[p - 1] for p in order_set]


def _gate_pack_backward(ctx, gG, H, C, gate_w, alpha, props):
    """pack backward -> transposed k-hop propagation -> hop-gate backward, the
    last one adding the pack's and the propagation's gradients into
    (grad H_norm, grad C_norm) in the same pass."""
    D = ctx.D
    gH, gC, gP, gA = _pack.pack_backward(gG.contiguous(), H, C, props, alpha, *PACK_MODES,
                                         need_alpha=True)
    grads = [None] * max(ctx.order_set)
    for p, g in zip(ctx.order_set, gP):
        grads[p - 1] = g
    del gP
    gHC = ctx.plan.backward(grads, 2 * D)  # dL/d[H | C] through the propagation
    del grads
    add_c = _lib.c_void_p(gHC.data_ptr() + D * gHC.element_size())  # right half
    gw, gb = hop_gate_backward_raw(H, C, gate_w, alpha, gA, ctx.gate_mode, gH, gC,
                                   accumulate=True, add_h=_lib.ptr(gHC), add_c=add_c,
                                   add_ld=2 * D)
    return gH, gC, gw, gb


def propagate_gate_pack_proj_forward_raw(H, C, gate_w, gate_b, proj_w, proj_b, plan, order_set,
                                         gate_mode, keep_g):
    """Forward of _PropagateGatePackProjFn on contiguous H, C: (out, saved) with
    saved = [H, C, gate_w, alpha, proj_w, *props] (+ [G] when kept), the
    tensors propagate_gate_pack_proj_backward_raw reads."""
    props = _propagate(H, C, plan, order_set)
    D, K = H.size(1), len(props)
    fused = (not keep_g) if USE_TCGEN05_PACK_PROJ is None else USE_TCGEN05_PACK_PROJ
    if (fused and torch.backends.cuda.matmul.allow_tf32
            and _pack.pack_proj_supported(D, K, proj_w.size(0))):
        alpha = hop_gate_forward_raw(H, C, gate_w, gate_b, gate_mode)
        out, G = _pack.pack_proj_forward(H, C, props, alpha, proj_w, proj_b, keep_g)
    else:
        G, alpha = _gate_pack(H, C, props, gate_w, gate_b, gate_mode)
        out = torch.addmm(proj_b, G, proj_w.t())
        if not keep_g:
            G = None
    saved = [H, C, gate_w, alpha, proj_w, *props]
    if G is not None:
        saved.append(G)
    return out, saved


class _NodeState:
    """The non-tensor state a propagate/gate/pack backward reads (the ctx
    attributes of the autograd nodes that run it)."""

    def __init__(self, plan, order_set, gate_mode, D):
        self.plan, self.order_set, self.gate_mode, self.D = plan, tuple(order_set), gate_mode, D


def propagate_gate_pack_proj_backward_raw(saved, g, plan, order_set, gate_mode):
    """Backward of _PropagateGatePackProjFn from its saved tensors:
    (gH, gC, g_gate_w, g_gate_b, g_proj_w, g_proj_b).  gH is a fresh tensor
    written by the hop-gate backward (callers may accumulate into it)."""
    H, C, gate_w, alpha, proj_w, *rest = saved
    K = len(order_set)
    props = rest[:K]
    g = g.contiguous()
    G = rest[K] if len(rest) > K else _pack.pack_forward(H, C, props, alpha, *PACK_MODES)
    g_proj_w = _weight_grad(g, G)
    del G
    g_proj_b = colsum(g)
    gG = g.mm(proj_w)
    state = _NodeState(plan, order_set, gate_mode, H.size(1))
    gH, gC, gw, gb = _gate_pack_backward(state, gG, H, C, gate_w, alpha, props)
    return gH, gC, gw, gb, g_proj_w, g_proj_b


class _PropagateGatePackProjFn(torch.autograd.Function):
    """The same node followed by the block's proj linear layer.

    With TF32 matmuls allowed (torch.backends.cuda.matmul.allow_tf32) and
    supported shapes, pack and proj run as one tcgen05 GEMM whose A operand
    is the pack, evaluated tile by tile in shared memory
    (cign_pack_proj_gemm_tf32); otherwise as the pack kernel and an fp32
    addmm.  keep_g=False (graphs where G_raw [N, 2KD] is too large to keep)
    stores no G_raw: the backward recomputes it (one pack pass, bit-identical)
    for the proj weight gradient."""

    @staticmethod
    def forward(ctx, H, C, gate_w, gate_b, proj_w, proj_b, plan, order_set, gate_mode, keep_g):
        out, saved = propagate_gate_pack_proj_forward_raw(
            H.contiguous(), C.contiguous(), gate_w, gate_b, proj_w, proj_b, plan, order_set,
            gate_mode, keep_g)
        ctx.save_for_backward(*saved)
        ctx.plan, ctx.order_set, ctx.gate_mode = plan, tuple(order_set), gate_mode
        return out

    @staticmethod
    def backward(ctx, g):
        gH, gC, gw, gb, g_proj_w, g_proj_b = propagate_gate_pack_proj_backward_raw(
            list(ctx.saved_tensors), g, ctx.plan, ctx.order_set, ctx.gate_mode)
        return gH, gC, gw, gb, g_proj_w, g_proj_b, None, None, None, None


def propagate_gate_pack(H_norm: torch.Tensor, C_norm: torch.Tensor, gate_w: torch.Tensor,
                        gate_b: torch.Tensor, plan: SpmmPlan, order_set: Sequence[int],
                        score_mode: str) -> torch.Tensor:
    order = tuple(int(p) for p in order_set)
    if len(set(order)) != len(order) or min(order) < 1:
        raise ValueError("order_set must hold distinct positive hop counts")
    return _PropagateGatePackFn.apply(H_norm, C_norm, gate_w, gate_b, plan, order,
                                      1 if score_mode == "new" else 0)


def propagate_gate_pack_proj(H_norm: torch.Tensor, C_norm: torch.Tensor, gate_w: torch.Tensor,
                             gate_b: torch.Tensor, plan: SpmmPlan, order_set: Sequence[int],
                             score_mode: str, proj_w: torch.Tensor, proj_b: torch.Tensor,
                             keep_g: bool = True) -> torch.Tensor:
    """linear(propagate_gate_pack(...), proj_w, proj_b) as one node; keep_g=False
    recomputes G_raw in the backward instead of keeping it."""
    order = tuple(int(p) for p in order_set)
    if len(set(order)) != len(order) or min(order) < 1:
        raise ValueError("order_set must hold distinct positive hop counts")
    return _PropagateGatePackProjFn.apply(H_norm, C_norm, gate_w, gate_b, proj_w, proj_b, plan,
                                          order, 1 if score_mode == "new" else 0, bool(keep_g))
