"""Torch-CPU restatement of every hot-path op -- TEST INFRASTRUCTURE.

Forward math is written out from the reference; gradients come from torch
autograd on these forward restatements (the reference's own CPU-runnable
oracles do the same: validate_*.py compare fused ops against autograd of
plain torch expressions).  All functions take CPU tensors.
"""
from __future__ import annotations

from typing import Dict, Optional, Sequence

import torch
import torch.nn.functional as F

from . import rng


# --------------------------------------------------------------------- SpMM
def csr_tensor(crow, col, val, n_rows: int, n_cols: int) -> torch.Tensor:
    """CSR(P) as a torch CPU tensor, the form prepare_fixed_csr_operator
    caches (model.py:149-186)."""
    return torch.sparse_csr_tensor(torch.as_tensor(crow, dtype=torch.int64),
                                   torch.as_tensor(col, dtype=torch.int64),
                                   torch.as_tensor(val, dtype=torch.float32),
                                   size=(n_rows, n_cols))


class _FixedSpMM(torch.autograd.Function):
    """Y = P X, grad_X = P^T grad_Y: FixedCSRSpMMFunction (model.py:57-106),
    with CPU torch.sparse.mm."""

    @staticmethod
    def forward(ctx, x, P, PT):
        ctx.PT = PT
        return torch.sparse.mm(P, x)

    @staticmethod
    def backward(ctx, g):
        return torch.sparse.mm(ctx.PT, g.contiguous()), None, None


def spmm(P, PT, x):
    """fixed_sparse_mm: one application of P (model.py:189-192)."""
    return _FixedSpMM.apply(x, P, PT)


def multihop(P, PT, x, powers) -> Dict[int, torch.Tensor]:
    """dict{p: P^p x} by recurrence (multihop_csr_pipeline.py:233-246 and
    model.py:247-252); backward through the recurrence is the reference's
    acc = P^T (acc + g_p) chain (:248-265)."""
    requested = sorted(set(int(p) for p in powers))
    out = {}
    if 0 in requested:
        out[0] = x
    cur = x
    for p in range(1, max(requested) + 1):
        cur = spmm(P, PT, cur)
        if p in requested:
            out[p] = cur
    return out


# ---------------------------------------------------------------------- GAT
def gat_collapsed(attn_row, attn_col, rowptr, col, in_feat, bias, negative_slope: float,
                  attn_drop: float, seed: int):
    """Collapsed GAT forward (collapsed_gat_cuda.cu:52-174, mask :34-47):
    per destination row i and head h over CSR edges e = (i, j):
      e_ij = leaky(attn_row[i,h] + attn_col[j,h]); m = max_e, s = sum exp(e - m);
      w = keep(e*H+h) * exp(e - m) / s / (1 - p);
      pre = sum_h sum_e w * in_feat[j,h,:] / H + bias;  out = SiLU(pre).
    Returns (out, pre, edge_max, edge_sum).  Rows without edges get
    max = -1e38, sum = 0 and out = SiLU(bias)."""
    n, H, C = in_feat.shape
    rowptr = torch.as_tensor(rowptr, dtype=torch.int64)
    col = torch.as_tensor(col, dtype=torch.int64)
    nnz = int(col.numel())
    deg = rowptr[1:] - rowptr[:-1]
    row = torch.repeat_interleave(torch.arange(n), deg)
    logit = F.leaky_relu(attn_row[row] + attn_col[col], negative_slope)       # [nnz, H]
    init = torch.full((n, H), -1.0e38, dtype=logit.dtype)
    m = init.scatter_reduce(0, row[:, None].expand(-1, H), logit.detach(), reduce="amax",
                            include_self=True)
    ex = torch.exp(logit - m[row])
    s = torch.zeros((n, H), dtype=logit.dtype).index_add(0, row, ex)
    safe_s = torch.where(s > 0, s, torch.ones_like(s))
    w = ex / safe_s[row]
    w = torch.where((s > 0)[row], w, torch.zeros_like(w))
    if attn_drop > 0.0:
        keep = torch.from_numpy(rng.gat_keep_mask(seed, nnz * H, attn_drop).reshape(nnz, H))
        w = torch.where(keep, w / (1.0 - attn_drop), torch.zeros_like(w))
    acc = torch.zeros((n, C), dtype=in_feat.dtype)
    for h in range(H):  # per head keeps the [nnz, C] message tensor small
        acc = acc.index_add(0, row, w[:, h, None] * in_feat[col, h, :])
    pre = acc / H + bias
    return F.silu(pre), pre, m.detach(), s.detach()


def gatconv_mean_bias_silu(x, att_src, att_dst, edge_index_src_dst, bias, negative_slope):
    """Independent formulation used only to cross-check gat_collapsed:
    PyG GATConv(concat=False, add_self_loops=False) message passing on a
    source->target edge list (per-target softmax over incoming edges,
    dropout off), head mean, bias, SiLU (model.py:472-480).  Softmax is taken
    with torch.softmax over each target's dense incoming-logit row."""
    n, H, C = x.shape
    a_src = (x * att_src).sum(-1)
    a_dst = (x * att_dst).sum(-1)
    src = torch.as_tensor(edge_index_src_dst[0], dtype=torch.int64)
    dst = torch.as_tensor(edge_index_src_dst[1], dtype=torch.int64)
    out = torch.zeros((n, H, C), dtype=x.dtype)
    for i in range(n):
        sel = dst == i
        if not bool(sel.any()):
            continue
        j = src[sel]
        logits = F.leaky_relu(a_dst[i][None, :] + a_src[j], negative_slope)   # [k, H]
        alpha = torch.softmax(logits, dim=0)
        out[i] = (alpha[:, :, None] * x[j]).sum(0)
    return F.silu(out.mean(1) + bias)


def attention_logits(x, att_src, att_dst):
    """alpha_src, alpha_dst = (x * att).sum(-1)  (validate_a3v3.py:38-39)."""
    return (x * att_src).sum(dim=-1), (x * att_dst).sum(dim=-1)


def head_mean_bias_silu(out, bias):
    """SiLU(mean_h out + bias)  (validate_a3v3.py:72)."""
    return F.silu(out.mean(dim=1) + bias)


# --------------------------------------------------------------------- pack
def pack(H, C, props: Sequence[torch.Tensor], alpha: Optional[torch.Tensor], interaction: str,
         outer: str, weighting: str):
    """Clifford pack family: validate_a3.py:8-19 legacy_pack (old interaction),
    validate_cign_switch_pack.py:17-50 (tanh switch) and
    validate_cign_acceleration.py:10-18 (CIGN, no outer nonlinearity)."""
    Ds, Ws = [], []
    for P in props:
        TH, TC = P.split(H.size(1), dim=-1)
        bhr = H * TC
        brh = C * TH
        if interaction == "old":
            Ds.append(F.silu(bhr))
            Ws.append(bhr - brh)
        else:
            Ds.append(F.silu(0.5 * (bhr + brh)))
            raw = 0.5 * (bhr - brh)
            Ws.append(torch.tanh(raw) if outer == "tanh" else raw)
    D = torch.stack(Ds, dim=1)
    W = torch.stack(Ws, dim=1)
    if alpha is None:
        alpha = torch.ones(H.size(0), len(props), dtype=H.dtype)
    if alpha.dim() == 3:
        alpha = alpha.squeeze(-1)
    A = alpha.unsqueeze(-1)
    if weighting == "old":
        return (torch.cat([W, D], dim=-1) * A).reshape(H.size(0), -1)
    return torch.cat([(D * A).sum(1), (W * A).sum(1)], dim=-1)


# ---------------------------------------------------------------- block ops
def _block_dropout(x, p: float, seed: int):
    if p <= 0.0:
        return x
    keep = torch.from_numpy(rng.block_keep_mask(seed, x.numel(), p).reshape(x.shape))
    return torch.where(keep, x * (1.0 / (1.0 - p)), torch.zeros_like(x))


def dropout_layernorm(x, w, b, p: float, eps: float, seed: int):
    """LN(dropout(x)) with the block-op mask (fused_block_ops.py:15
    dropout_ln_forward_kernel; validate_a3v8.py:27-31 for p = 0)."""
    return F.layer_norm(_block_dropout(x, p, seed), (x.size(1),), w, b, eps)


def add_layernorm(a, b, w, bias, eps: float):
    """LN(a + b) (generic_engine/validate_a3v8.py:29; fused_add_layernorm,
    fused_block_ops.py:112)."""
    return F.layer_norm(a + b, (a.size(1),), w, bias, eps)


def dropout_gamma_residual(h, g, gamma, p: float, seed: int):
    """h + gamma * dropout(g) (validate_a3v8.py:30)."""
    return h + gamma.unsqueeze(0) * _block_dropout(g, p, seed)
