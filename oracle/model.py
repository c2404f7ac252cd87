"""CIGN model on the CPU oracle ops -- TEST INFRASTRUCTURE.

A restatement of generic_engine/model_cign.py's GraphCliffordNet in the
production configuration (local_train.py:5: alpha score "new", interaction
"new", weighting "old", outer nonlinearity "none"; hop gate "node", gamma
"vector", JK "concat", dual input projection) written with the unfused
torch expressions of the reference's fallback branches
(model_cign.py:758-937, 1160-1212) and the oracle ops.  Parameter names are
the reference's, so a state_dict from cign_b200.model_cign loads as is.

Used by the model parity tests and as the CPU baseline of bench.py.
Dropout inside the oracle ops uses the reference's splitmix64 streams;
the input/output dropouts use torch's CPU RNG (as F.dropout does in the
reference), so parity tests run with dropout 0.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops, rng


class OracleGAT(nn.Module):
    """GATConv(concat=False) + bias + SiLU on the collapsed-GAT restatement
    (CompatibleCollapsedFusedGATConv.forward, generic_engine/model_cign.py:524-570)."""

    def __init__(self, in_channels, out_channels, heads, dropout, negative_slope=0.2):
        super().__init__()
        self.heads, self.out_channels = heads, out_channels
        self.dropout, self.negative_slope = dropout, negative_slope
        self.lin = nn.Linear(in_channels, heads * out_channels, bias=False)
        self.att_src = nn.Parameter(torch.zeros(1, heads, out_channels))
        self.att_dst = nn.Parameter(torch.zeros(1, heads, out_channels))
        self.bias = nn.Parameter(torch.zeros(out_channels))

    def forward(self, x, gat_graph, seed: int):
        xh = self.lin(x).view(-1, self.heads, self.out_channels)
        a_src, a_dst = ops.attention_logits(xh, self.att_src, self.att_dst)
        (rowptr, col), _, _ = gat_graph
        p = self.dropout if self.training else 0.0
        out, _, _, _ = ops.gat_collapsed(a_dst, a_src, rowptr, col, xh, self.bias,
                                         self.negative_slope, p, seed)
        return out


class OracleBlock(nn.Module):
    """GraphCliffordBlock with every fused switch off
    (generic_engine/model_cign.py:573-937)."""

    def __init__(self, hidden_dim, order_set, dropout, gat_heads, gat_dropout, init_gamma=0.49):
        super().__init__()
        self.hidden_dim = hidden_dim
        self.order_set = [int(s) for s in order_set]
        self.num_hops = len(self.order_set)
        self.dropout = dropout
        self.h_norm = nn.LayerNorm(hidden_dim)
        self.c_norm = nn.LayerNorm(hidden_dim)
        self.context_gat = OracleGAT(hidden_dim, hidden_dim, gat_heads, gat_dropout)
        self.proj = nn.Linear(2 * self.num_hops * hidden_dim, hidden_dim, bias=True)
        self.hop_gate_mlp = nn.Linear(2 * hidden_dim, self.num_hops, bias=True)
        self.gamma = nn.Parameter(torch.full((hidden_dim,), float(init_gamma)))

    def forward(self, H, P, PT, gat_graph, seeds):
        p = self.dropout if self.training else 0.0
        H_norm = ops.dropout_layernorm(H, self.h_norm.weight, self.h_norm.bias, p, self.h_norm.eps,
                                       seeds["ln"])
        C_gat = self.context_gat(H_norm, gat_graph, seeds["gat"])
        C_norm = ops.add_layernorm(C_gat, H_norm, self.c_norm.weight, self.c_norm.bias,
                                   self.c_norm.eps)
        HC = torch.cat([H_norm, C_norm], dim=-1)
        prop = ops.multihop(P, PT, HC, self.order_set)
        gate_input = torch.cat([H_norm + C_norm, torch.abs(H_norm - C_norm)], dim=-1)
        alpha = F.softmax(self.hop_gate_mlp(gate_input), dim=-1).unsqueeze(-1)
        G_raw = ops.pack(H_norm, C_norm, [prop[s] for s in self.order_set], alpha, "new", "none",
                         "old")
        G_feat = self.proj(G_raw)
        return ops.dropout_gamma_residual(H, G_feat, self.gamma, p, seeds["res"])


class OracleCIGN(nn.Module):
    """GraphCliffordNet: dual input projection, blocks, JK concat, LayerNorm,
    classifier (generic_engine/model_cign.py:943-1215)."""

    def __init__(self, in_dim, hidden_dim, out_dim, num_layers, order_set, dropout, gat_heads,
                 gat_dropout, init_gamma=0.49, init_input_eta=0.1):
        super().__init__()
        self.dropout = dropout
        self.input_proj_0 = nn.Linear(in_dim, hidden_dim, bias=True)
        self.input_proj_1 = nn.Linear(in_dim, hidden_dim, bias=True)
        self.input_eta = nn.Parameter(torch.tensor(float(init_input_eta)))
        self.blocks = nn.ModuleList([
            OracleBlock(hidden_dim, order_set, dropout, gat_heads, gat_dropout, init_gamma)
            for _ in range(num_layers)
        ])
        final_dim = hidden_dim * (num_layers + 1)
        self.output_norm = nn.LayerNorm(final_dim)
        self.classifier = nn.Linear(final_dim, out_dim, bias=True)
        self.calls = 0

    def forward(self, x, P, PT, gat_graph, initial_seed: int = 0, gat_call0: int = 0,
                block_call0: int = 0):
        """Seeds follow the reference's per-call counters: one GAT counter and
        one shared block-op counter (tags 1 and 2), advanced only when the
        corresponding dropout is active.  gat_call0 / block_call0 are the
        counters' values before this forward (0 for a fresh process)."""
        x = x.float()
        H_in = F.dropout(x, p=self.dropout, training=self.training)
        H = F.silu(self.input_proj_0(H_in)) + self.input_eta * F.silu(self.input_proj_1(H_in))
        states = [H]
        gat_call = int(gat_call0)
        block_call = int(block_call0)
        for blk in self.blocks:
            p = blk.dropout if self.training else 0.0
            gp = blk.context_gat.dropout if self.training else 0.0
            seeds = {}
            if p > 0:
                block_call += 1
                seeds["ln"] = rng.block_seed(initial_seed, block_call, 1)
            else:
                seeds["ln"] = 0
            if gp > 0:
                seeds["gat"] = rng.gat_seed(initial_seed, gat_call)
                gat_call += 1
            else:
                seeds["gat"] = 0
            if p > 0:
                block_call += 1
                seeds["res"] = rng.block_seed(initial_seed, block_call, 2)
            else:
                seeds["res"] = 0
            H = blk(H, P, PT, gat_graph, seeds)
            states.append(H)
        H_out = self.output_norm(torch.cat(states, dim=-1))
        H_out = F.dropout(H_out, p=self.dropout, training=self.training)
        return self.classifier(H_out)
