"""A whole CIGN block as one autograd node (generic_engine/model_cign.py:759-929,
production switches, unpartitioned graph):

    H_norm = dropout-LayerNorm(H)                          (h_norm)
    lin    = GAT context of H_norm up to its bias          (aggregate-first)
    C_norm = LayerNorm(SiLU(lin + bias) + H_norm)          (c_norm)
    G_feat = proj(pack(H_norm, C_norm, P^p [H_norm | C_norm], hop gate))
    out    = H + gamma * dropout(G_feat)

Composed op by op, autograd sums the gradients of H_norm (three consumers:
the GAT context, the add-LayerNorm and the propagation/gate/pack node) and
of H (the LayerNorm and the residual) with separate add kernels, each a full
read-read-write pass over an [N, D] tensor.  Here the backward writes each
of those gradients once and lets the later producers add into it in their
own passes:

* the hop-gate backward writes grad H_norm (pack + propagation + gate);
* the SiLU/add-LayerNorm backward adds its share in place
  (cign_silu_add_ln_bwd, accumulate_z);
* the GAT context adds gfeat @ W by a beta = 1 GEMM and its logit term in
  place (cign_row_dots_bwd);
* the dropout-LayerNorm backward adds the residual's gradient as it writes
  grad H (cign_dropout_ln_bwd_add).

Forward values, dropout streams (seed draw order: block dropout-LN, GAT,
block residual) and parameter gradients are those of the op-by-op block.
"""
from __future__ import annotations

import torch

from . import collapsed_gat as _gat
from . import fused_block_ops as _blk
from .block_fused import (native_spmm_plan, propagate_gate_pack_proj_backward_raw,
                          propagate_gate_pack_proj_forward_raw)


class _BlockConfig:
    """Non-tensor arguments of one block call."""

    __slots__ = ("p", "ln_eps", "cn_eps", "ln_seed", "gat_seed", "res_seed", "gat_plan",
                 "heads", "n_dst", "att_shape", "slope", "attn_drop", "spmm_plan", "order_set",
                 "gate_mode", "keep_g")

    def __init__(self, **kw):
        for k, v in kw.items():
            setattr(self, k, v)


class _CignBlockFn(torch.autograd.Function):
    """The block's tensors for the backward are kept as attributes of ctx,
    not through save_for_backward, so that the backward can drop each group
    as soon as its last consumer has run (the propagation's hop outputs, for
    instance, before the GAT backward allocates its workspace) instead of
    holding all of them until the node returns.  None of them is an output
    of this node, so no reference cycle arises.  Unlike save_for_backward,
    this does not detect an in-place change of the block input or of a
    parameter between the forward and the backward (a training step makes
    none: the optimizer runs after the backward); such a change would give
    wrong gradients instead of an error."""

    @staticmethod
    def forward(ctx, H, ln_w, ln_b, gat_w, att_src, att_dst, gat_bias, cn_w, cn_b, gate_w,
                gate_b, proj_w, proj_b, gamma, cfg):
        H = H.contiguous()
        H_norm, ln_mean, ln_rstd = _blk.dropout_ln_forward(H, ln_w, ln_b, cfg.p, cfg.ln_eps,
                                                           cfg.ln_seed)
        lin, gat_saved = _gat.gat_context_lin_forward_raw(
            H_norm, gat_w, att_src, att_dst, cfg.gat_plan, cfg.heads, cfg.n_dst, cfg.slope,
            cfg.attn_drop, cfg.gat_seed)
        C_norm, pre, cn_mean, cn_rstd = _gat.silu_add_ln_forward(lin, gat_bias, H_norm, cn_w, cn_b,
                                                                 cfg.cn_eps)
        del lin
        G_feat, prop_saved = propagate_gate_pack_proj_forward_raw(
            H_norm, C_norm, gate_w, gate_b, proj_w, proj_b, cfg.spmm_plan, cfg.order_set,
            cfg.gate_mode, cfg.keep_g)
        out = _blk.gamma_residual_forward(H, G_feat, gamma, cfg.p, cfg.res_seed)
        ctx.cfg = cfg
        ctx.ln = (H, ln_w, ln_mean, ln_rstd)
        ctx.gat = (gat_w, gat_saved)
        ctx.cn = (pre, cn_w, cn_mean, cn_rstd)
        ctx.res = (G_feat, gamma)
        ctx.prop = prop_saved  # starts with (H_norm, C_norm, gate_w)
        return out

    @staticmethod
    def backward(ctx, g_out):
        cfg = ctx.cfg
        g_out = g_out.to(torch.float32).contiguous()
        G_feat, gamma = ctx.res
        del ctx.res
        gG, g_gamma = _blk.gamma_residual_backward(g_out, G_feat, gamma, cfg.p, cfg.res_seed)
        del G_feat
        prop_saved = ctx.prop
        del ctx.prop
        H_norm = prop_saved[0]
        gH_norm, gC_norm, g_gate_w, g_gate_b, g_proj_w, g_proj_b = \
            propagate_gate_pack_proj_backward_raw(prop_saved, gG, cfg.spmm_plan, cfg.order_set,
                                                  cfg.gate_mode)
        del prop_saved, gG
        # the add-LayerNorm's share of grad H_norm, added in place
        pre, cn_w, cn_mean, cn_rstd = ctx.cn
        del ctx.cn
        _, g_lin, g_cn_w, g_cn_b, g_gat_bias = _gat.silu_add_ln_backward(
            gC_norm, pre, H_norm, cn_w, cn_mean, cn_rstd, grad_h=gH_norm)
        del gC_norm, pre
        # the GAT context's share, added in place
        gat_w, gat_saved = ctx.gat
        del ctx.gat
        _, g_gat_w, g_att_src, g_att_dst = _gat.gat_context_lin_backward_raw(
            H_norm, gat_w, gat_saved, g_lin, cfg.gat_plan, cfg.heads, cfg.n_dst, cfg.att_shape,
            cfg.slope, cfg.attn_drop, cfg.gat_seed, grad_x=gH_norm)
        del g_lin, gat_saved, H_norm
        # grad H = LayerNorm backward + the residual branch's g_out, one pass
        H, ln_w, ln_mean, ln_rstd = ctx.ln
        del ctx.ln
        g_H, g_ln_w, g_ln_b = _blk.dropout_ln_backward(gH_norm, H, ln_w, ln_mean, ln_rstd, cfg.p,
                                                       cfg.ln_seed, addend=g_out)
        return (g_H, g_ln_w, g_ln_b, g_gat_w, g_att_src, g_att_dst, g_gat_bias, g_cn_w, g_cn_b,
                g_gate_w, g_gate_b, g_proj_w, g_proj_b, g_gamma, None)


def block_node_applies(block, H, graph_operator, gat_graph) -> bool:
    """Whether cign_block can run `block` on these inputs: CUDA fp32 [N, D]
    with D % 4 == 0 and D <= 1024, an unpartitioned GAT graph triple, the
    aggregate-first GAT, a native k-hop operator and the production pack
    switches (those of the fused propagate/gate/pack/proj node)."""
    D = H.size(1) if H.dim() == 2 else -1
    gat = block.context_gat
    return (H.is_cuda and H.dtype == torch.float32 and H.dim() == 2 and D % 4 == 0
            and D <= _blk.MAX_D and isinstance(gat_graph, (tuple, list))
            and gat.aggregate_first and gat.out_channels % 4 == 0 and gat.out_channels == D
            and block.interaction_mode == "new" and block.outer_nonlinearity == "none"
            and block.alpha_weighting_mode == "old" and block.alpha_score_mode in ("new", "old")
            and block.num_hops <= 8 and len(set(block.order_set)) == block.num_hops
            and min(block.order_set) >= 1
            and not getattr(graph_operator, "is_row_partitioned", False)
            and native_spmm_plan(graph_operator) is not None)


def cign_block(block, H: torch.Tensor, graph_operator, gat_graph) -> torch.Tensor:
    """block(H) (GraphCliffordBlock.forward) as one autograd node; the caller
    checks block_node_applies first."""
    p = block.dropout if block.training else 0.0
    gat = block.context_gat
    attn_drop = gat.dropout if block.training else 0.0
    csr, csc, perm = gat_graph
    # seeds drawn in the op-by-op block's order
    ln_seed = _blk._next_seed(1, p)
    gat_plan, heads, n_dst = _gat._gat_context_args(H, gat.lin.weight, gat.att_src, gat.att_dst,
                                                    csr, csc, perm, attn_drop, H.size(0))
    gat_seed = _gat.gat_call_seed(attn_drop)
    res_seed = _blk._next_seed(2, p)
    cfg = _BlockConfig(p=float(p), ln_eps=float(block.h_norm.eps), cn_eps=float(block.c_norm.eps),
                       ln_seed=ln_seed, gat_seed=gat_seed, res_seed=res_seed, gat_plan=gat_plan,
                       heads=int(heads), n_dst=int(n_dst), att_shape=gat.att_src.shape,
                       slope=float(gat.negative_slope), attn_drop=float(attn_drop),
                       spmm_plan=native_spmm_plan(graph_operator),
                       order_set=tuple(block.order_set),
                       gate_mode=1 if block.alpha_score_mode == "new" else 0,
                       keep_g=not block._recompute_pack(H))
    return _CignBlockFn.apply(H, block.h_norm.weight, block.h_norm.bias, gat.lin.weight,
                              gat.att_src, gat.att_dst, gat.bias, block.c_norm.weight,
                              block.c_norm.bias, block.hop_gate_mlp.weight,
                              block.hop_gate_mlp.bias, block.proj.weight, block.proj.bias,
                              block.gamma, cfg)
