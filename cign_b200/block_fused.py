"""The middle of a CIGN block as one autograd node:

    HC     = [H_norm | C_norm]
    T^p    = P^p HC,  p in order_set                 (k-hop propagation)
    alpha  = softmax(hop_gate([H+C, |H-C|]))         (hop gate)
    G_raw  = Clifford pack(H_norm, C_norm, T, alpha)

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

from typing import Optional, Sequence

import torch

from . import _lib, _pack
from .hop_gate import hop_gate_backward_raw, hop_gate_forward_raw
from .multihop_csr_pipeline import (GenericMultiHopCSRGraphOperator,
                                    HybridNative3TailCSRGraphOperator, MultiHopCSR3GraphOperator)
from .plans import SpmmPlan, spmm_plan_for

PACK_MODES = (1, 0, 0)  # interaction "new", outer none, weighting "old"


def native_spmm_plan(operator) -> Optional[SpmmPlan]:
    """The SpmmPlan behind a k-hop operator of multihop_csr_pipeline (None for
    other operators, e.g. a row-partitioned one)."""
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
        max_power = max(order_set)
        ys = plan.forward(torch.cat([H, C], 1), max_power)
        props = [ys[p - 1] for p in order_set]
        alpha = hop_gate_forward_raw(H, C, gate_w, gate_b, gate_mode)
        G = _pack.pack_forward(H, C, props, alpha, *PACK_MODES)
        ctx.save_for_backward(H, C, gate_w, alpha, *props)
        ctx.plan, ctx.order_set, ctx.gate_mode, ctx.D = plan, tuple(order_set), gate_mode, D
        return G

    @staticmethod
    def backward(ctx, gG):
        H, C, gate_w, alpha, *props = ctx.saved_tensors
        D = ctx.D
        gH, gC, gP, gA = _pack.pack_backward(gG.contiguous(), H, C, props, alpha, *PACK_MODES,
                                             need_alpha=True)
        grads = [None] * max(ctx.order_set)
        for p, g in zip(ctx.order_set, gP):
            grads[p - 1] = g
        gHC = ctx.plan.backward(grads, 2 * D)  # dL/d[H | C] through the propagation
        add_c = _lib.c_void_p(gHC.data_ptr() + D * gHC.element_size())  # right half
        gw, gb = hop_gate_backward_raw(H, C, gate_w, alpha, gA, ctx.gate_mode, gH, gC,
                                       accumulate=True, add_h=_lib.ptr(gHC), add_c=add_c,
                                       add_ld=2 * D)
        return gH, gC, gw, gb, None, None, None


def propagate_gate_pack(H_norm: torch.Tensor, C_norm: torch.Tensor, gate_w: torch.Tensor,
                        gate_b: torch.Tensor, plan: SpmmPlan, order_set: Sequence[int],
                        score_mode: str) -> torch.Tensor:
    order = tuple(int(p) for p in order_set)
    if len(set(order)) != len(order) or min(order) < 1:
        raise ValueError("order_set must hold distinct positive hop counts")
    return _PropagateGatePackFn.apply(H_norm, C_norm, gate_w, gate_b, plan, order,
                                      1 if score_mode == "new" else 0)
