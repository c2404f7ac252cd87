"""CIGN (Graph Clifford network) on the native hot path.

The reference's generic_engine/model_cign.py is the unchanged caller of the
hot-path modules; this module restates its fused configuration so the full
training step can run where the reference tree is absent (benchmarks, GPU
tests).  Parameter names and shapes are the reference's (PyG GATConv
`lin`/`att_src`/`att_dst`/`bias`, block `h_norm`/`c_norm`/`proj`/
`hop_gate_mlp`/`gamma`, net `input_proj_0/1`/`input_eta`/`output_norm`/
`classifier`), so state dicts move between the two.

Block forward (model_cign.py:751-937, production switches of
local_train.py:5 -- alpha score "new", interaction "new", weighting "old",
outer nonlinearity "none"):
    H_norm = dropout_LN(H)                                  fused_block_ops
    x      = lin(H_norm).view(N, heads, D)                  cuBLAS (TF32)
    a_s, a_d = attention logits(x)                          fused_gat_sideops
    C_gat  = SiLU(mean_h GAT(x) + bias)                     collapsed_gat
    C_norm = LN(C_gat + H_norm)                             fused_block_ops
  (GATContext evaluates the GAT aggregate-first by default:
   a = H_norm @ (W_h^T att)^T, z_h = GAT-weighted sums of H_norm rows,
   lin = z @ M -- the same function with lin applied after the aggregation,
   so each edge gathers one D-float row, not heads*D -- and the block then
   forms C_norm = LN(SiLU(lin + bias) + H_norm) in one pass,
   gat_silu_add_layernorm, without storing C_gat.)
    T^k    = P^k [H_norm | C_norm], k in order_set          multihop_csr_pipeline
    alpha  = softmax(hop_gate_mlp([H+C | |H-C|]))           hop_gate (fused)
    G_raw  = Clifford pack(H_norm, C_norm, T, alpha)        fused_clifford_*
    H'     = H + gamma * dropout(proj(G_raw))               fused_block_ops
On an unpartitioned graph with these switches the whole block runs as one
autograd node (block_node.cign_block), whose backward accumulates the
gradients of H_norm and H in-kernel instead of with separate add passes.
Net (model_cign.py:1160-1212): dropout, dual input projection + SiLU, L
blocks, JK concat, LayerNorm, dropout, classifier.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import fused_clifford_cign_generic, fused_clifford_cign_pack, fused_clifford_pack
from .collapsed_gat import (collapsed_gat_mean_bias_silu, gat_context, gat_context_lin,
                            gat_silu_add_layernorm)
from .fused_block_ops import fused_add_layernorm, fused_dropout_gamma_residual, fused_dropout_layernorm
from .fused_gat_sideops import fused_attention_logits
from .graph_operator import selected_sparse_powers
from .input_proj import dual_input_projection
from .block_fused import native_spmm_plan, propagate_gate_pack_proj
from .block_node import block_node_applies, cign_block
from .jk_norm import jk_layer_norm, jk_norm_supported
from .hop_gate import fused_hop_gate
from .linear import linear


def _glorot_(t: torch.Tensor) -> None:
    fan_in, fan_out = t.size(-2), t.size(-1)
    a = math.sqrt(6.0 / (fan_in + fan_out))
    with torch.no_grad():
        t.uniform_(-a, a)


def _linear_padded(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """F.linear with the output width padded to a multiple of 4 (zero rows of
    weight/bias) and sliced back: a 5-wide output row is not 16-byte aligned,
    which sends cuBLAS to slow unaligned kernels; the padded columns are
    never read, so values and gradients equal F.linear's."""
    k = weight.size(0)
    pad = (-k) % 4
    if pad == 0 or not x.is_cuda:
        return F.linear(x, weight, bias)
    w = F.pad(weight, (0, 0, 0, pad))
    b = F.pad(bias, (0, pad))
    return F.linear(x, w, b)[:, :k]


class GATContext(nn.Module):
    """Parameters of PyG GATConv(in, out, heads, concat=False, bias=True):
    lin [heads*out, in] (no bias), att_src/att_dst [1, heads, out], bias [out]."""

    def __init__(self, in_channels: int, out_channels: int, heads: int, dropout: float,
                 negative_slope: float = 0.2):
        super().__init__()
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.heads = heads
        self.dropout = dropout
        self.negative_slope = negative_slope
        self.concat = False
        self.lin = nn.Linear(in_channels, heads * out_channels, bias=False)
        self.att_src = nn.Parameter(torch.empty(1, heads, out_channels))
        self.att_dst = nn.Parameter(torch.empty(1, heads, out_channels))
        self.bias = nn.Parameter(torch.zeros(out_channels))
        # evaluate lin after the aggregation (same function, 4x fewer gathered
        # bytes per edge at H=4); False keeps the lin -> collapsed-GAT order
        self.aggregate_first = True
        _glorot_(self.lin.weight)
        _glorot_(self.att_src)
        _glorot_(self.att_dst)

    def forward_lin(self, x: torch.Tensor, gat_graph):
        """The head-mean GAT output before its bias and SiLU ([N, C]) when the
        aggregate-first form applies, else None; the block then evaluates
        bias + SiLU + add-LayerNorm in one op (gat_silu_add_layernorm)."""
        H, C = self.heads, self.out_channels
        if not (self.aggregate_first and x.size(1) % 4 == 0 and C % 4 == 0):
            return None
        drop = self.dropout if self.training else 0.0
        if hasattr(gat_graph, "halo"):  # cign_b200.distributed.DistGatGraph
            csr, csc, perm = gat_graph.csr, gat_graph.csc, gat_graph.perm
            x_src = gat_graph.halo(x)
        else:
            csr, csc, perm = gat_graph
            x_src = x
        return gat_context_lin(x_src, self.lin.weight, self.att_src, self.att_dst, csr, csc, perm,
                               self.negative_slope, drop, n_dst=x.size(0))

    def forward(self, x: torch.Tensor, gat_graph) -> torch.Tensor:
        H, C = self.heads, self.out_channels
        drop = self.dropout if self.training else 0.0
        partitioned = hasattr(gat_graph, "halo")  # cign_b200.distributed.DistGatGraph
        if partitioned:
            csr, csc, perm = gat_graph.csr, gat_graph.csc, gat_graph.perm
            x_src = gat_graph.halo(x)  # own rows, then the halo rows from their owners
        else:
            csr, csc, perm = gat_graph
            x_src = x
        if self.aggregate_first and x.size(1) % 4 == 0 and C % 4 == 0:
            # lin is linear: aggregate x per head, apply lin.weight afterwards;
            # alpha_src[n,h] = <W_h x_n, att_src[h]> = <x_n, W_h^T att_src[h]>.
            return gat_context(x_src, self.lin.weight, self.att_src, self.att_dst, self.bias, csr,
                               csc, perm, self.negative_slope, drop, n_dst=x.size(0))
        if partitioned:
            raise NotImplementedError("a partitioned graph needs the aggregate-first GAT form")
        xh = self.lin(x).view(-1, H, C)
        a_src, a_dst = fused_attention_logits(xh, self.att_src, self.att_dst)
        return collapsed_gat_mean_bias_silu(
            attn_row=a_dst, attn_col=a_src, csr=csr, csc=csc, perm=perm,
            negative_slope=self.negative_slope, in_feat=xh, bias=self.bias,
            attn_drop=drop,
        )


class GraphCliffordBlock(nn.Module):
    def __init__(self, hidden_dim: int, order_set=(1, 2, 3), dropout: float = 0.28,
                 gat_heads: int = 6, gat_dropout: float = 0.32, init_gamma: float = 0.49,
                 alpha_score_mode: str = "new", interaction_mode: str = "new",
                 alpha_weighting_mode: str = "old", outer_nonlinearity: str = "none"):
        super().__init__()
        if len(order_set) == 0:
            raise ValueError("order_set / hop_scales cannot be empty.")
        self.hidden_dim = hidden_dim
        self.order_set = [int(s) for s in order_set]
        self.num_hops = len(self.order_set)
        self.dropout = dropout
        self.alpha_score_mode = alpha_score_mode
        self.interaction_mode = interaction_mode
        self.alpha_weighting_mode = alpha_weighting_mode
        self.outer_nonlinearity = outer_nonlinearity
        self.h_norm = nn.LayerNorm(hidden_dim)
        self.c_norm = nn.LayerNorm(hidden_dim)
        self.context_gat = GATContext(hidden_dim, hidden_dim, gat_heads, gat_dropout)
        proj_in = 2 * self.num_hops * hidden_dim if alpha_weighting_mode == "old" else 2 * hidden_dim
        self.proj = nn.Linear(proj_in, hidden_dim, bias=True)
        self.hop_gate_mlp = nn.Linear(2 * hidden_dim, self.num_hops, bias=True)
        self.gamma = nn.Parameter(torch.full((hidden_dim,), float(init_gamma)))

    # G_raw [N, 2*K*D] at or above this size is recomputed in the backward
    # instead of being kept (None: decide by size; True/False: always/never)
    recompute_pack = None
    RECOMPUTE_PACK_BYTES = 4 << 30

    def _recompute_pack(self, H_norm) -> bool:
        if self.recompute_pack is not None:
            return bool(self.recompute_pack)
        return H_norm.size(0) * 2 * self.num_hops * self.hidden_dim * 4 >= self.RECOMPUTE_PACK_BYTES

    def compute_hop_gate(self, H_norm, C_norm):
        if H_norm.size(1) % 4 == 0 and self.num_hops <= 8 and H_norm.is_cuda:
            return fused_hop_gate(H_norm, C_norm, self.hop_gate_mlp.weight, self.hop_gate_mlp.bias,
                                  self.alpha_score_mode).unsqueeze(-1)
        if self.alpha_score_mode == "old":
            gate_input = torch.cat([H_norm, C_norm], dim=-1)
        else:
            gate_input = torch.cat([H_norm + C_norm, torch.abs(H_norm - C_norm)], dim=-1)
        return F.softmax(self.hop_gate_mlp(gate_input), dim=-1).unsqueeze(-1)

    # run the whole block as one autograd node where it applies
    # (cign_b200.block_node: gradients accumulated in-kernel, no add passes)
    use_block_node = True

    def forward(self, H, graph_operator, gat_graph):
        if (self.use_block_node and native_spmm_plan(graph_operator) is not None
                and block_node_applies(self, H, graph_operator, gat_graph)):
            return cign_block(self, H, graph_operator, gat_graph)
        p = self.dropout if self.training else 0.0
        H_norm = fused_dropout_layernorm(H, self.h_norm.weight, self.h_norm.bias, p, self.h_norm.eps)
        lin = self.context_gat.forward_lin(H_norm, gat_graph)
        if lin is not None:
            # GAT bias + SiLU and the add-LayerNorm in one pass (forward and backward)
            C_norm = gat_silu_add_layernorm(lin, self.context_gat.bias, H_norm, self.c_norm.weight,
                                            self.c_norm.bias, self.c_norm.eps)
        else:
            C_gat = self.context_gat(H_norm, gat_graph)
            C_norm = fused_add_layernorm(C_gat, H_norm, self.c_norm.weight, self.c_norm.bias,
                                         self.c_norm.eps)
        plan = native_spmm_plan(graph_operator)
        if (plan is not None and self.interaction_mode == "new" and self.outer_nonlinearity == "none"
                and self.alpha_weighting_mode == "old" and self.alpha_score_mode in ("new", "old")
                and H_norm.size(1) % 4 == 0 and self.num_hops <= 8
                and len(set(self.order_set)) == self.num_hops and min(self.order_set) >= 1):
            # propagation + hop gate + pack as one node (gradients merged in-kernel)
            args = (H_norm, C_norm, self.hop_gate_mlp.weight, self.hop_gate_mlp.bias, plan,
                    self.order_set, self.alpha_score_mode)
            G_feat = propagate_gate_pack_proj(*args, self.proj.weight, self.proj.bias,
                                              keep_g=not self._recompute_pack(H_norm))
            return fused_dropout_gamma_residual(H, G_feat, self.gamma, p)
        HC = torch.cat([H_norm, C_norm], dim=-1)
        propagated = selected_sparse_powers(graph_operator, HC, self.order_set)
        hop_gate = self.compute_hop_gate(H_norm, C_norm)
        props = [propagated[s] for s in self.order_set]
        if self.interaction_mode == "old":
            G_raw = fused_clifford_pack.fused_clifford_pack(H_norm, C_norm, props, hop_gate)
            if self.alpha_weighting_mode == "new":
                packed = G_raw.reshape(H.size(0), self.num_hops, 2 * self.hidden_dim)
                G_raw = torch.cat([packed[..., self.hidden_dim:].sum(1),
                                   packed[..., :self.hidden_dim].sum(1)], dim=-1)
        elif self.outer_nonlinearity == "none" and self.num_hops == 3:
            G_raw = fused_clifford_cign_pack.fused_clifford_switch_pack(
                H_norm, C_norm, props, hop_gate, "new", self.alpha_weighting_mode)
        elif self.outer_nonlinearity == "none":
            G_raw = fused_clifford_cign_generic.fused_clifford_pack(H_norm, C_norm, props, hop_gate)
            if self.alpha_weighting_mode == "new":
                packed = G_raw.reshape(H.size(0), self.num_hops, 2 * self.hidden_dim)
                G_raw = torch.cat([packed[..., self.hidden_dim:].sum(1),
                                   packed[..., :self.hidden_dim].sum(1)], dim=-1)
        else:
            from .fused_clifford_switch_pack import fused_clifford_switch_pack
            G_raw = fused_clifford_switch_pack(H_norm, C_norm, props, hop_gate, "new",
                                               self.alpha_weighting_mode)
        G_feat = linear(G_raw, self.proj.weight, self.proj.bias)
        return fused_dropout_gamma_residual(H, G_feat, self.gamma, p)


class GraphCliffordNet(nn.Module):
    def __init__(self, in_dim: int, hidden_dim: int, out_dim: int, num_layers: int = 4,
                 order_set=(1, 2, 3), dropout: float = 0.28, gat_heads: int = 6,
                 gat_dropout: float = 0.32, init_gamma: float = 0.49, init_input_eta: float = 0.1,
                 alpha_score_mode: str = "new", interaction_mode: str = "new",
                 alpha_weighting_mode: str = "old", outer_nonlinearity: str = "none"):
        super().__init__()
        if num_layers <= 0:
            raise ValueError("num_layers must be positive.")
        self.dropout = dropout
        self.num_layers = num_layers
        self.hidden_dim = hidden_dim
        self.input_act = nn.SiLU()
        self.input_proj_0 = nn.Linear(in_dim, hidden_dim, bias=True)
        self.input_proj_1 = nn.Linear(in_dim, hidden_dim, bias=True)
        self.input_eta = nn.Parameter(torch.tensor(float(init_input_eta)))
        self.blocks = nn.ModuleList([
            GraphCliffordBlock(hidden_dim, order_set, dropout, gat_heads, gat_dropout, init_gamma,
                               alpha_score_mode, interaction_mode, alpha_weighting_mode,
                               outer_nonlinearity)
            for _ in range(num_layers)
        ])
        final_dim = hidden_dim * (num_layers + 1)
        self.output_norm = nn.LayerNorm(final_dim)
        self.classifier = nn.Linear(final_dim, out_dim, bias=True)
        self._gat_graph = None

    def prepare_fused_gat_graph(self, gat_graph) -> None:
        """Set the ((rowptr, col), (row, colptr), perm) triple used by every block."""
        self._gat_graph = gat_graph

    def forward(self, x: torch.Tensor, graph_operator) -> torch.Tensor:
        if self._gat_graph is None:
            raise RuntimeError("call prepare_fused_gat_graph(...) once before training")
        x = x.float()
        H_in = F.dropout(x, p=self.dropout, training=self.training)
        if H_in.is_cuda and self.hidden_dim % 4 == 0 and not H_in.requires_grad:
            # both projections in one GEMM, SiLU and the eta mix in one pass
            H = dual_input_projection(H_in, self.input_proj_0.weight, self.input_proj_0.bias,
                                      self.input_proj_1.weight, self.input_proj_1.bias,
                                      self.input_eta)
        else:
            H = self.input_act(linear(H_in, self.input_proj_0.weight, self.input_proj_0.bias)) + \
                self.input_eta * self.input_act(linear(H_in, self.input_proj_1.weight,
                                                       self.input_proj_1.bias))
        states = [H]
        for block in self.blocks:
            H = block(H, graph_operator, self._gat_graph)
            states.append(H)
        if jk_norm_supported(states):  # LayerNorm of the cat, without the cat
            H_out = jk_layer_norm(states, self.output_norm.weight, self.output_norm.bias,
                                  self.output_norm.eps)
        else:
            H_out = self.output_norm(torch.cat(states, dim=-1))
        H_out = F.dropout(H_out, p=self.dropout, training=self.training)
        return _linear_padded(H_out, self.classifier.weight, self.classifier.bias).float()


def build_model(in_dim: int, hidden_dim: int, out_dim: int, num_layers: int = 4,
                dropout: float = 0.28, hop_scales=(1, 2, 3), gat_heads: int = 6,
                gat_dropout: float = 0.32, **kwargs) -> GraphCliffordNet:
    """Factory with the reference's argument names (model_cign.py:1217-1278);
    the use_fused_* switches are accepted and ignored (always native)."""
    keep = {k: kwargs[k] for k in ("init_gamma", "init_input_eta", "alpha_score_mode",
                                   "interaction_mode", "alpha_weighting_mode",
                                   "outer_nonlinearity") if k in kwargs and kwargs[k] is not None}
    return GraphCliffordNet(in_dim, hidden_dim, out_dim, num_layers, hop_scales, dropout, gat_heads,
                            gat_dropout, **keep)
