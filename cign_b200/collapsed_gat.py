"""Collapsed multi-head GAT core (drop-in for the reference's collapsed_gat).

``collapsed_gat_mean_bias_silu(attn_row, attn_col, csr, csc, perm,
negative_slope, in_feat, bias, attn_drop)`` computes, for destination row i,
``SiLU(mean_h sum_j w_ijh in_feat[j,h,:] + bias)`` with
``w = dropout(softmax_j(LeakyReLU(attn_row[i,h] + attn_col[j,h])))``
(collapsed_gat.py:164-225; kernels collapsed_gat_ext/collapsed_gat_cuda.cu).
Gradients flow to attn_row, attn_col, in_feat and bias; graph tensors get
None (collapsed_gat.py:148-161).

The dropout stream matches the reference bit for bit: per call the seed is
``(initial_seed & (2^63-1)) + 0x9E3779B97F4A7C15 * (call_id + 1)`` modulo 2^63
with a module-level call counter that does not advance when attn_drop == 0
(collapsed_gat.py:201-211), and the keep bit of (CSR edge e, head h) is the
splitmix64 Bernoulli of index e*H + h.  The mask is recomputed in backward
rather than stored.  Unlike the reference kernel (H=6, C=256 only,
collapsed_gat.cpp:67-68) any 1 <= H <= 64 and C >= 1 run natively.
"""
from __future__ import annotations

import contextlib

import torch

from . import _lib, seeds
from .plans import gat_plan_for

_EXT = None
_EXT_ERROR = None
_CALL_COUNTER = seeds.counter_iter(seeds.GAT)  # GAT call ids (shared with seeds.next_seed)
MAX_HEADS = 64


def _extension_name() -> str:
    return "cign_sm100_collapsed_gat"


def ensure_collapsed_gat_loaded(verbose: bool = False):
    global _EXT, _EXT_ERROR
    if _EXT is not None:
        return _EXT
    if _EXT_ERROR is not None:
        raise RuntimeError("collapsed GAT extension previously failed to load") from _EXT_ERROR
    if not torch.cuda.is_available():
        raise RuntimeError("A3-v6 collapsed GAT requires CUDA")
    try:
        _EXT = _lib.load_library()
    except Exception as exc:
        _EXT_ERROR = exc
        raise
    return _EXT


def gat_call_seed(attn_drop: float):
    """Seed of the next call (advances the counter only when attn_drop > 0):
    an int, or a device seed slot while a seeds.DeviceSeedTable records."""
    return seeds.next_seed(seeds.GAT, attn_drop)


def gat_forward_raw(plan, attn_row, attn_col, in_feat, bias, negative_slope, attn_drop, seed):
    """Native forward; returns (out, pre, edge_max, edge_sum)."""
    lib = ensure_collapsed_gat_loaded()
    n, H, C = (int(s) for s in in_feat.shape)
    out = torch.empty((n, C), dtype=torch.float32, device=in_feat.device)
    pre = torch.empty_like(out)
    emax = torch.empty((n, H), dtype=torch.float32, device=in_feat.device)
    esum = torch.empty_like(emax)
    ws = _lib.workspace(lib.cign_gat_fwd_workspace_bytes(plan.handle, H, C), in_feat.device)
    with _lib.DeviceGuard(in_feat.device):
        rc = lib.cign_gat_fwd(plan.handle, H, C, _lib.ptr(attn_row), _lib.ptr(attn_col),
                              _lib.ptr(in_feat), _lib.ptr(bias), float(negative_slope),
                              float(attn_drop), *_lib.seed_args(seed), _lib.ptr(out),
                              _lib.ptr(pre), _lib.ptr(emax), _lib.ptr(esum), _lib.ptr(ws),
                              ws.numel(), _lib.stream_of(in_feat))
    _lib.check(rc, "cign_gat_fwd")
    return out, pre, emax, esum


def gat_backward_raw(plan, attn_row, attn_col, in_feat, pre, emax, esum, grad_y, negative_slope,
                     attn_drop, seed):
    """Native backward; returns (grad_feat, grad_attn_row, grad_attn_col, grad_bias)."""
    lib = ensure_collapsed_gat_loaded()
    n, H, C = (int(s) for s in in_feat.shape)
    dev = in_feat.device
    gfeat = torch.empty_like(in_feat)
    grow = torch.empty((n, H), dtype=torch.float32, device=dev)
    gcol = torch.empty_like(grow)
    gbias = torch.empty((C,), dtype=torch.float32, device=dev)
    nbytes = int(lib.cign_gat_bwd_workspace_bytes(plan.handle, H, C))
    ws = _lib.workspace(nbytes, dev)
    with _lib.DeviceGuard(dev):
        rc = lib.cign_gat_bwd(plan.handle, H, C, _lib.ptr(attn_row), _lib.ptr(attn_col),
                              _lib.ptr(in_feat), _lib.ptr(pre), _lib.ptr(emax), _lib.ptr(esum),
                              _lib.ptr(grad_y), float(negative_slope), float(attn_drop),
                              *_lib.seed_args(seed), _lib.ptr(gfeat), _lib.ptr(grow),
                              _lib.ptr(gcol), _lib.ptr(gbias), _lib.ptr(ws), ws.numel(),
                              _lib.stream_of(in_feat))
    _lib.check(rc, "cign_gat_bwd")
    return gfeat, grow, gcol, gbias


def gat_dropout_mask(nnz: int, heads: int, attn_drop: float, seed: int, device) -> torch.Tensor:
    """uint8 [nnz, H] keep-mask of one call (parity checks only)."""
    lib = ensure_collapsed_gat_loaded()
    mask = torch.empty((int(nnz), int(heads)), dtype=torch.uint8, device=device)
    with _lib.DeviceGuard(device):
        rc = lib.cign_gat_dropout_mask(int(nnz), int(heads), float(attn_drop),
                                       *_lib.seed_args(seed), _lib.ptr(mask),
                                       _lib.stream_on(device))
    _lib.check(rc, "cign_gat_dropout_mask")
    return mask


class _CollapsedGATFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, attn_row, attn_col, rowptr, col, colptr, row, perm, negative_slope, in_feat,
                bias, attn_drop, seed):
        ensure_collapsed_gat_loaded(False)
        attn_row = attn_row.contiguous()
        attn_col = attn_col.contiguous()
        in_feat = in_feat.contiguous()
        bias = bias.contiguous()
        plan = gat_plan_for(rowptr, col, row, colptr, perm)
        n, H, C = in_feat.shape
        if tuple(attn_row.shape) != (n, H) or tuple(attn_col.shape) != (n, H):
            raise RuntimeError("attn_row/attn_col must be [N,H] matching in_feat")
        if bias.dim() != 1 or bias.size(0) != C:
            raise RuntimeError("bias must be [C]")
        if plan.n != n:
            raise RuntimeError(f"graph has {plan.n} rows but in_feat has {n}")
        out, pre, emax, esum = gat_forward_raw(plan, attn_row, attn_col, in_feat, bias,
                                               negative_slope, attn_drop, seed)
        ctx.save_for_backward(attn_row, attn_col, in_feat, pre, emax, esum)
        ctx.plan = plan
        ctx.negative_slope = float(negative_slope)
        ctx.attn_drop = float(attn_drop)
        ctx.seed = seed
        return out

    @staticmethod
    def backward(ctx, grad_y):
        attn_row, attn_col, in_feat, pre, emax, esum = ctx.saved_tensors
        gfeat, grow, gcol, gbias = gat_backward_raw(
            ctx.plan, attn_row, attn_col, in_feat, pre, emax, esum,
            grad_y.to(torch.float32).contiguous(), ctx.negative_slope, ctx.attn_drop, ctx.seed)
        return grow, gcol, None, None, None, None, None, None, gfeat, gbias, None, None


def collapsed_gat_mean_bias_silu(
    attn_row: torch.Tensor,
    attn_col: torch.Tensor,
    csr,
    csc,
    perm: torch.Tensor,
    negative_slope: float,
    in_feat: torch.Tensor,
    bias: torch.Tensor,
    attn_drop: float,
) -> torch.Tensor:
    if in_feat.dtype != torch.float32 or in_feat.device.type != "cuda":
        raise TypeError("A3-v6 collapsed GAT requires CUDA float32 in_feat")
    if bias is None:
        raise ValueError("A3-v6 collapsed GAT currently requires bias=True")
    if in_feat.dim() != 3:
        raise ValueError(f"in_feat must be [N,H,C], got {tuple(in_feat.shape)}")
    H = int(in_feat.size(1))
    if not (1 <= H <= MAX_HEADS):
        raise ValueError(f"collapsed GAT requires 1<=H<={MAX_HEADS}; got H={H}")
    if not (0.0 <= float(attn_drop) < 1.0):
        raise ValueError("attn_drop must be in [0,1)")
    (rowptr, col), (row, colptr) = csr, csc
    seed = gat_call_seed(attn_drop)
    return _CollapsedGATFn.apply(attn_row, attn_col, rowptr, col, colptr, row, perm,
                                 float(negative_slope), in_feat, bias, float(attn_drop), seed)


# ---------------------------------------------------------------- aggregate-first
def gat_agg_forward_raw(plan, attn_row, attn_col, x, heads, negative_slope, attn_drop, seed):
    """z [N,H,D] fp32 = per-head attention-weighted sums of x rows; returns
    (z, emax, esum).  x may be float32 or bfloat16 (bf16 storage, widened to
    fp32 as it is gathered: cign_gat_agg_fwd_bf16, D % 8 == 0)."""
    lib = ensure_collapsed_gat_loaded()
    D = int(x.size(1))
    n = int(plan.n)  # destination rows (x has plan.n_cols rows)
    H = int(heads)
    z = torch.empty((n, H, D), dtype=torch.float32, device=x.device)
    emax = torch.empty((n, H), dtype=torch.float32, device=x.device)
    esum = torch.empty_like(emax)
    ws = _lib.workspace(lib.cign_gat_agg_workspace_bytes(plan.handle, H, D, D), x.device)
    fn, name = ((lib.cign_gat_agg_fwd_bf16, "cign_gat_agg_fwd_bf16") if x.dtype == torch.bfloat16
                else (lib.cign_gat_agg_fwd, "cign_gat_agg_fwd"))
    with _lib.DeviceGuard(x.device):
        rc = fn(plan.handle, H, D, _lib.ptr(attn_row), _lib.ptr(attn_col), _lib.ptr(x),
                float(negative_slope), float(attn_drop), *_lib.seed_args(seed), _lib.ptr(z),
                _lib.ptr(emax), _lib.ptr(esum), _lib.ptr(ws), ws.numel(), _lib.stream_of(x))
    _lib.check(rc, name)
    return z, emax, esum


def gat_agg_forward_keep_raw(plan, attn_row, attn_col, x, heads, negative_slope, attn_drop,
                             seed):
    """gat_agg_forward_raw on fp32 x that also returns the edge weights
    [nnz, H] (cign_gat_agg_fwd_w): (z, emax, esum, wts), wts to be handed to
    gat_agg_backward_raw so that the backward does not form them again."""
    lib = ensure_collapsed_gat_loaded()
    D = int(x.size(1))
    n = int(plan.n)
    H = int(heads)
    z = torch.empty((n, H, D), dtype=torch.float32, device=x.device)
    emax = torch.empty((n, H), dtype=torch.float32, device=x.device)
    esum = torch.empty_like(emax)
    wts = torch.empty((max(int(plan.nnz), 1), H), dtype=torch.float32, device=x.device)
    ws = _lib.workspace(lib.cign_gat_agg_workspace_bytes(plan.handle, H, D, D), x.device)
    with _lib.DeviceGuard(x.device):
        rc = lib.cign_gat_agg_fwd_w(plan.handle, H, D, _lib.ptr(attn_row), _lib.ptr(attn_col),
                                    _lib.ptr(x), float(negative_slope), float(attn_drop),
                                    *_lib.seed_args(seed), _lib.ptr(z), _lib.ptr(emax),
                                    _lib.ptr(esum), _lib.ptr(wts), _lib.ptr(ws), ws.numel(),
                                    _lib.stream_of(x))
    _lib.check(rc, "cign_gat_agg_fwd_w")
    return z, emax, esum, wts


def gat_agg_backward_raw(plan, attn_row, attn_col, x, emax, esum, grad_z, grad_pre, negative_slope,
                         attn_drop, seed, wts=None):
    """Returns (grad_feat [N,H,C], grad_attn_row [N,H], grad_attn_col [N,H]).
    With wts (the forward's edge weights, gat_agg_forward_keep_raw) the
    backward reads them instead of forming them again."""
    lib = ensure_collapsed_gat_loaded()
    n_cols, D = (int(s) for s in x.shape)
    n = int(plan.n)
    H = int(emax.size(1))
    C = int(grad_pre.size(1))
    dev = x.device
    gfeat = torch.empty((n_cols, H, C), dtype=torch.float32, device=dev)
    grow = torch.empty((n, H), dtype=torch.float32, device=dev)
    gcol = torch.empty((n_cols, H), dtype=torch.float32, device=dev)
    ws = _lib.workspace(lib.cign_gat_agg_workspace_bytes(plan.handle, H, D, C), dev)
    with _lib.DeviceGuard(dev):
        if wts is None:
            rc = lib.cign_gat_agg_bwd(plan.handle, H, D, C, _lib.ptr(attn_row),
                                      _lib.ptr(attn_col), _lib.ptr(x), _lib.ptr(emax),
                                      _lib.ptr(esum), _lib.ptr(grad_z), _lib.ptr(grad_pre),
                                      float(negative_slope), float(attn_drop),
                                      *_lib.seed_args(seed), _lib.ptr(gfeat), _lib.ptr(grow),
                                      _lib.ptr(gcol), _lib.ptr(ws), ws.numel(), _lib.stream_of(x))
            name = "cign_gat_agg_bwd"
        else:
            rc = lib.cign_gat_agg_bwd_w(plan.handle, H, D, C, _lib.ptr(attn_row),
                                        _lib.ptr(attn_col), _lib.ptr(x), _lib.ptr(emax),
                                        _lib.ptr(esum), _lib.ptr(grad_z), _lib.ptr(grad_pre),
                                        _lib.ptr(wts), float(negative_slope), float(attn_drop),
                                        *_lib.seed_args(seed), _lib.ptr(gfeat), _lib.ptr(grow),
                                        _lib.ptr(gcol), _lib.ptr(ws), ws.numel(),
                                        _lib.stream_of(x))
            name = "cign_gat_agg_bwd_w"
    _lib.check(rc, name)
    return gfeat, grow, gcol


def _bias_silu(lin: torch.Tensor, bias: torch.Tensor):
    """(SiLU(lin + bias), lin + bias) in one pass (cign_head_mean_bias_silu_fwd, 1 head)."""
    lib = ensure_collapsed_gat_loaded()
    n, C = (int(s) for s in lin.shape)
    out = torch.empty_like(lin)
    pre = torch.empty_like(lin)
    with _lib.DeviceGuard(lin.device):
        rc = lib.cign_head_mean_bias_silu_fwd(n, 1, C, _lib.ptr(lin), _lib.ptr(bias.contiguous()),
                                              _lib.ptr(out), _lib.ptr(pre), _lib.stream_of(lin))
    _lib.check(rc, "cign_head_mean_bias_silu_fwd")
    return out, pre


def _bias_silu_backward(grad_out: torch.Tensor, pre: torch.Tensor):
    """(g_pre = grad_out * SiLU'(pre), fixed-order column sums of g_pre)."""
    lib = ensure_collapsed_gat_loaded()
    grad_out = grad_out.to(torch.float32).contiguous()
    n, C = (int(s) for s in pre.shape)
    g_pre = torch.empty_like(pre)
    g_bias = torch.empty((C,), dtype=torch.float32, device=pre.device)
    ws = _lib.workspace(lib.cign_head_mean_bias_silu_bwd_workspace_bytes(n, C), pre.device)
    with _lib.DeviceGuard(pre.device):
        rc = lib.cign_head_mean_bias_silu_bwd(n, 1, C, _lib.ptr(grad_out), _lib.ptr(pre),
                                              _lib.ptr(g_pre), _lib.ptr(g_bias), _lib.ptr(ws),
                                              ws.numel(), _lib.stream_of(pre))
    _lib.check(rc, "cign_head_mean_bias_silu_bwd")
    return g_pre, g_bias


def _head_projection(weight: torch.Tensor, heads: int) -> torch.Tensor:
    """M [H*D, C] with M[(h,d), c] = W[h*C + c, d] / H, so that
    z.view(N, H*D) @ M = (1/H) sum_h W_h z[:, h, :]."""
    HC, D = weight.shape
    C = HC // heads
    return weight.view(heads, C, D).permute(0, 2, 1).reshape(heads * D, C) / heads


class _AggregateFirstLinFn(torch.autograd.Function):
    """lin = mean_h sum_j w_ijh (lin.weight_h x_j), computed as z.view(N, H*D) @ M
    with z = cign_gat_agg_fwd(x): the collapsed GAT's head-mean output before
    its bias (collapsed_gat_cuda.cu:52-174 with in_feat = lin(x)).

    z is not kept for the backward: the weight gradient sum_i z_i^T g_i
    equals sum_j gfeat_j^T x_j (gfeat = the gradient of lin(x).view(N,H,C),
    which the backward kernels produce anyway), so only x is saved."""

    @staticmethod
    def forward(ctx, x, attn_row, attn_col, weight, plan, heads, negative_slope, attn_drop,
                seed):
        H = int(heads)
        n, D = int(plan.n), int(x.size(1))
        z, emax, esum = gat_agg_forward_raw(plan, attn_row, attn_col, x, H, negative_slope,
                                            attn_drop, seed)
        M = _head_projection(weight, H)
        lin = z.view(n, H * D).mm(M)
        del z
        ctx.save_for_backward(x, attn_row, attn_col, weight, emax, esum)
        ctx.plan, ctx.heads = plan, H
        ctx.negative_slope, ctx.attn_drop, ctx.seed = float(negative_slope), float(attn_drop), seed
        return lin

    @staticmethod
    def backward(ctx, g_lin):
        x, attn_row, attn_col, weight, emax, esum = ctx.saved_tensors
        H = ctx.heads
        n_cols = int(x.size(0))
        C = weight.size(0) // H
        g_pre = g_lin.contiguous()
        M = _head_projection(weight, H)
        grad_z = g_pre.mm(M.t())                                    # [N, H*D]
        gfeat, grow, gcol = gat_agg_backward_raw(ctx.plan, attn_row, attn_col, x, emax, esum,
                                                 grad_z, g_pre, ctx.negative_slope,
                                                 ctx.attn_drop, ctx.seed)
        del grad_z
        gfeat2 = gfeat.view(n_cols, H * C)
        grad_w = gfeat2.t().mm(x)                                   # [H*C, D]
        grad_x = gfeat2.mm(weight)                                  # [N_cols, D]
        return grad_x, grow, gcol, grad_w, None, None, None, None, None


class _BiasSiLUFn(torch.autograd.Function):
    """SiLU(lin + bias) (the collapsed GAT's epilogue, collapsed_gat_cuda.cu:167-173)."""

    @staticmethod
    def forward(ctx, lin, bias):
        out, pre = _bias_silu(lin, bias)
        ctx.save_for_backward(pre)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        (pre,) = ctx.saved_tensors
        g_pre, grad_bias = _bias_silu_backward(grad_out, pre)
        return g_pre, grad_bias


def aggregate_first_with_plan(x, attn_row, attn_col, weight, bias, plan, heads, negative_slope,
                              attn_drop, seed):
    """SiLU(lin + bias) of the aggregate-first GAT on an existing plan (the
    body of collapsed_gat_aggregate_first, for callers holding a plan)."""
    lin = _AggregateFirstLinFn.apply(x, attn_row, attn_col, weight, plan, heads, negative_slope,
                                     attn_drop, seed)
    return _BiasSiLUFn.apply(lin, bias)


def silu_add_ln_forward(lin, bias, h, weight, ln_bias, eps):
    """(y, pre, mean, rstd) of cign_silu_add_ln_fwd."""
    lib = ensure_collapsed_gat_loaded()
    n, D = (int(v) for v in lin.shape)
    y = torch.empty_like(lin)
    pre = torch.empty_like(lin)
    mean = torch.empty((n,), dtype=torch.float32, device=lin.device)
    rstd = torch.empty_like(mean)
    with _lib.DeviceGuard(lin.device):
        rc = lib.cign_silu_add_ln_fwd(n, D, _lib.ptr(lin), _lib.ptr(bias), _lib.ptr(h),
                                      _lib.ptr(weight), _lib.ptr(ln_bias), float(eps),
                                      _lib.ptr(pre), _lib.ptr(y), _lib.ptr(mean), _lib.ptr(rstd),
                                      _lib.stream_of(lin))
    _lib.check(rc, "cign_silu_add_ln_fwd")
    return y, pre, mean, rstd


def silu_add_ln_backward(grad_y, pre, h, weight, mean, rstd, grad_h=None):
    """(grad_z, grad_pre, grad_w, grad_b, grad_bias) of cign_silu_add_ln_bwd.
    With grad_h given (h's gradient from its other consumers, [N, D]), grad_z
    is added into it in place and grad_h is returned as grad_z."""
    lib = ensure_collapsed_gat_loaded()
    n, D = (int(v) for v in pre.shape)
    acc = grad_h is not None
    if acc and (grad_h.shape != pre.shape or not grad_h.is_contiguous()):
        raise ValueError("grad_h must be a contiguous [N, D] tensor")
    gz = grad_h if acc else torch.empty_like(pre)
    gpre = torch.empty_like(pre)
    gw = torch.empty((D,), dtype=torch.float32, device=pre.device)
    gb = torch.empty_like(gw)
    gbias = torch.empty_like(gw)
    ws = _lib.workspace(lib.cign_silu_add_ln_bwd_workspace_bytes(n, D), pre.device)
    with _lib.DeviceGuard(pre.device):
        rc = lib.cign_silu_add_ln_bwd(n, D, _lib.ptr(grad_y), _lib.ptr(pre), _lib.ptr(h),
                                      _lib.ptr(weight), _lib.ptr(mean), _lib.ptr(rstd),
                                      int(acc), _lib.ptr(gz), _lib.ptr(gpre), _lib.ptr(gw),
                                      _lib.ptr(gb),
                                      _lib.ptr(gbias), _lib.ptr(ws), ws.numel(),
                                      _lib.stream_of(pre))
    _lib.check(rc, "cign_silu_add_ln_bwd")
    return gz, gpre, gw, gb, gbias


class _SiLUAddLayerNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, lin, bias, h, weight, ln_bias, eps):
        lin, h = lin.contiguous(), h.contiguous()
        y, pre, mean, rstd = silu_add_ln_forward(lin, bias, h, weight, ln_bias, eps)
        ctx.save_for_backward(pre, h, weight, mean, rstd)
        return y

    @staticmethod
    def backward(ctx, grad_y):
        pre, h, weight, mean, rstd = ctx.saved_tensors
        gz, gpre, gw, gb, gbias = silu_add_ln_backward(grad_y.contiguous(), pre, h, weight, mean,
                                                       rstd)
        return gpre, gbias, gz, gw, gb, None


def gat_silu_add_layernorm(lin: torch.Tensor, bias: torch.Tensor, h: torch.Tensor,
                           weight: torch.Tensor, ln_bias: torch.Tensor,
                           eps: float) -> torch.Tensor:
    """LayerNorm(SiLU(lin + bias) + h) with LayerNorm weight/ln_bias: the GAT
    layer's bias + SiLU epilogue and the block's add-LayerNorm
    (model_cign.py:767-787) as one op, forward and backward.  lin is the GAT's
    head-mean output before its bias (collapsed_gat_aggregate_first_lin)."""
    if lin.dim() != 2 or h.shape != lin.shape:
        raise ValueError("lin and h must both be [N, D]")
    return _SiLUAddLayerNormFn.apply(lin, bias, h, weight, ln_bias, float(eps))


@contextlib.contextmanager
def _full_fp32_matmul():
    """cuBLAS in full fp32 inside the block (TF32 off), the caller's setting after."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        yield
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def row_dots_forward(x: torch.Tensor, V: torch.Tensor) -> torch.Tensor:
    """out [N, K] = x [N, D] @ V[K, D]^T in fp32 (cign_row_dots_fwd)."""
    lib = ensure_collapsed_gat_loaded()
    n, D = (int(s) for s in x.shape)
    K = int(V.size(0))
    out = torch.empty((n, K), dtype=torch.float32, device=x.device)
    with _lib.DeviceGuard(x.device):
        rc = lib.cign_row_dots_fwd(n, D, K, _lib.ptr(x), _lib.ptr(V), _lib.ptr(out),
                                   _lib.stream_of(x))
    _lib.check(rc, "cign_row_dots_fwd")
    return out


def row_dots_backward(x: torch.Tensor, V: torch.Tensor, g: torch.Tensor, grad_x: torch.Tensor,
                      accumulate: bool) -> torch.Tensor:
    """grad_x (+)= g @ V in place; returns grad_V = g^T @ x (cign_row_dots_bwd)."""
    lib = ensure_collapsed_gat_loaded()
    n, D = (int(s) for s in x.shape)
    K = int(V.size(0))
    gV = torch.empty_like(V)
    ws = _lib.workspace(lib.cign_row_dots_bwd_workspace_bytes(n, D, K), x.device)
    with _lib.DeviceGuard(x.device):
        rc = lib.cign_row_dots_bwd(n, D, K, _lib.ptr(x), _lib.ptr(V), _lib.ptr(g),
                                   _lib.ptr(grad_x), 1 if accumulate else 0, _lib.ptr(gV),
                                   _lib.ptr(ws), ws.numel(), _lib.stream_of(x))
    _lib.check(rc, "cign_row_dots_bwd")
    return gV


def _logit_vectors(weight: torch.Tensor, att_src: torch.Tensor, att_dst: torch.Tensor,
                   heads: int):
    """(V [2H, D], A [H, 2, C]): V[h] = W_h^T att_src[h], V[H + h] = W_h^T att_dst[h]
    (W_h = weight[h*C:(h+1)*C]), in full fp32."""
    HC, D = (int(s) for s in weight.shape)
    H = int(heads)
    C = HC // H
    A = torch.cat([att_src.reshape(H, 1, C), att_dst.reshape(H, 1, C)], 1)
    with _full_fp32_matmul():
        V2 = torch.bmm(A, weight.view(H, C, D))                                  # [H, 2, D]
    return V2.transpose(0, 1).reshape(2 * H, D), A


def gat_context_lin_forward_raw(x, weight, att_src, att_dst, plan, heads, n_dst, negative_slope,
                                attn_drop, seed):
    """Forward of _GatContextLinFn: (lin [n_dst, C], saved) with saved the
    tensors its backward needs besides x and weight."""
    H = int(heads)
    V, A = _logit_vectors(weight, att_src, att_dst, H)
    alpha = row_dots_forward(x, V)                                                  # [N, 2H]
    attn_col = alpha[:, :H].contiguous()
    attn_row = alpha[:n_dst, H:].contiguous()
    n, D = int(plan.n), int(x.size(1))
    z, emax, esum, wts = gat_agg_forward_keep_raw(plan, attn_row, attn_col, x, H, negative_slope,
                                                  attn_drop, seed)
    M = _head_projection(weight, H)
    lin = z.view(n, H * D).mm(M)
    del z
    return lin, (attn_row, attn_col, emax, esum, V, A, wts)


def gat_context_lin_backward_raw(x, weight, saved, g_lin, plan, heads, n_dst, att_shape,
                                 negative_slope, attn_drop, seed, grad_x=None):
    """Backward of _GatContextLinFn: (grad_x, grad_w, grad_att_src, grad_att_dst).
    With grad_x given ([N_src, D], x's gradient from its other consumers) the
    GAT's share is added into it in place (beta = 1 GEMM, then the logit
    term), with no separate add."""
    attn_row, attn_col, emax, esum, V, A, wts = saved
    H = int(heads)
    n_src, D = (int(s) for s in x.shape)
    HC = int(weight.size(0))
    C = HC // H
    g_pre = g_lin.contiguous()
    M = _head_projection(weight, H)
    grad_z = g_pre.mm(M.t())                                                        # [N, H*D]
    gfeat, grow, gcol = gat_agg_backward_raw(plan, attn_row, attn_col, x, emax, esum, grad_z,
                                             g_pre, negative_slope, attn_drop, seed, wts=wts)
    del grad_z
    gfeat2 = gfeat.view(n_src, HC)
    if grad_x is None:
        grad_x = gfeat2.mm(weight)                                                  # [N_src, D]
    else:
        grad_x.addmm_(gfeat2, weight)
    g_alpha = torch.zeros((n_src, 2 * H), dtype=torch.float32, device=x.device)
    g_alpha[:, :H] = gcol
    g_alpha[:n_dst, H:] = grow
    gV = row_dots_backward(x, V, g_alpha, grad_x, accumulate=True)                  # [2H, D]
    gV2 = gV.view(2, H, D).transpose(0, 1)                                          # [H, 2, D]
    with _full_fp32_matmul():
        g_att = torch.bmm(weight.view(H, C, D), gV2.transpose(1, 2))                 # [H, C, 2]
        g_w_att = torch.bmm(A.transpose(1, 2), gV2)                                  # [H, C, D]
    grad_w = torch.addmm(g_w_att.reshape(HC, D), gfeat2.t(), x)                     # [H*C, D]
    g_src = g_att[:, :, 0].reshape(att_shape)
    g_dst = g_att[:, :, 1].reshape(att_shape)
    return grad_x, grad_w, g_src, g_dst


class _GatContextLinFn(torch.autograd.Function):
    """The GAT context of a CIGN block up to its bias: lin(x) -> attention
    logits (fused_gat_sideops.py:50-71) -> collapsed GAT head mean
    (collapsed_gat_cuda.cu:52-174) without its bias, as one node, evaluated
    aggregate-first (_AggregateFirstLinFn) with the logits as row dots of x
    with V = [W_h^T att_src[h] ; W_h^T att_dst[h]] (cign_row_dots_fwd): x is
    read once for all 2H logits and no [N, H*C] tensor is formed.  Rows
    [0, n_dst) of x are the destination rows (all of them unless the graph is
    a row-partitioned block with halo columns).

    Backward: the aggregation's gradients (gat_agg_backward_raw), then
    grad_x = gfeat W + g_alpha V with the second term added in place by
    cign_row_dots_bwd (no separate add), and grad W = gfeat^T x + the logit
    vectors' share.  The logits and their gradients stay in full fp32
    whatever the TF32 setting: the att_src / att_dst gradients are sums over
    every node of nearly cancelling terms."""

    @staticmethod
    def forward(ctx, x, weight, att_src, att_dst, plan, heads, n_dst, negative_slope, attn_drop,
                seed):
        lin, saved = gat_context_lin_forward_raw(x, weight, att_src, att_dst, plan, heads, n_dst,
                                                 negative_slope, attn_drop, seed)
        ctx.save_for_backward(x, weight, *saved)
        ctx.plan, ctx.heads, ctx.n_dst, ctx.att_shape = plan, int(heads), int(n_dst), att_src.shape
        ctx.negative_slope, ctx.attn_drop, ctx.seed = float(negative_slope), float(attn_drop), seed
        return lin

    @staticmethod
    def backward(ctx, g_lin):
        x, weight, *saved = ctx.saved_tensors
        grad_x, grad_w, g_src, g_dst = gat_context_lin_backward_raw(
            x, weight, saved, g_lin, ctx.plan, ctx.heads, ctx.n_dst, ctx.att_shape,
            ctx.negative_slope, ctx.attn_drop, ctx.seed)
        return grad_x, grad_w, g_src, g_dst, None, None, None, None, None, None


def _gat_context_args(x, weight, att_src, att_dst, csr, csc, perm, attn_drop, n_dst):
    if x.dtype != torch.float32 or x.device.type != "cuda" or x.dim() != 2:
        raise TypeError("aggregate-first GAT requires CUDA float32 x [N,D]")
    if att_src.dim() < 2:
        raise ValueError("att_src / att_dst must be [1, H, C]")
    H = int(att_src.size(-2))
    if not (1 <= H <= MAX_HEADS):
        raise ValueError(f"collapsed GAT requires 1<=H<={MAX_HEADS}; got H={H}")
    if weight.dim() != 2 or weight.size(0) % H != 0 or weight.size(1) != x.size(1):
        raise ValueError("weight must be [H*C, D]")
    C = weight.size(0) // H
    if att_src.numel() != H * C or att_dst.numel() != H * C:
        raise ValueError("att_src / att_dst must be [1, H, C]")
    if not (0.0 <= float(attn_drop) < 1.0):
        raise ValueError("attn_drop must be in [0,1)")
    (rowptr, col), (row, colptr) = csr, csc
    plan = gat_plan_for(rowptr, col, row, colptr, perm)
    n_dst = int(plan.n) if n_dst is None else int(n_dst)
    if plan.n_cols != x.size(0) or plan.n != n_dst:
        raise RuntimeError(f"graph is {plan.n} x {plan.n_cols} but x has {x.size(0)} rows "
                           f"({n_dst} destination rows)")
    return plan, H, n_dst


def gat_context_lin(x: torch.Tensor, weight: torch.Tensor, att_src: torch.Tensor,
                    att_dst: torch.Tensor, csr, csc, perm: torch.Tensor, negative_slope: float,
                    attn_drop: float, n_dst=None) -> torch.Tensor:
    """The head-mean GAT output before its bias ([n_dst, C]) of GATConv(x) with
    lin.weight = weight [H*C, D] and att_src / att_dst [1, H, C]: the logits,
    the segment softmax and the aggregation in one node (_GatContextLinFn).
    Pair it with gat_silu_add_layernorm or _BiasSiLUFn.  Same dropout stream
    (call counter and keep bits) as collapsed_gat_mean_bias_silu."""
    plan, H, n_dst = _gat_context_args(x, weight, att_src, att_dst, csr, csc, perm, attn_drop,
                                       n_dst)
    seed = gat_call_seed(attn_drop)
    return _GatContextLinFn.apply(x.contiguous(), weight, att_src, att_dst, plan, H, n_dst,
                                  float(negative_slope), float(attn_drop), seed)


def gat_context(x: torch.Tensor, weight: torch.Tensor, att_src: torch.Tensor,
                att_dst: torch.Tensor, bias: torch.Tensor, csr, csc, perm: torch.Tensor,
                negative_slope: float, attn_drop: float, n_dst=None) -> torch.Tensor:
    """SiLU(gat_context_lin(...) + bias): GATConv(concat=False) + bias + SiLU as
    collapsed_gat_mean_bias_silu computes it on lin(x)."""
    lin = gat_context_lin(x, weight, att_src, att_dst, csr, csc, perm, negative_slope, attn_drop,
                          n_dst)
    return _BiasSiLUFn.apply(lin, bias)


def collapsed_gat_aggregate_first(x: torch.Tensor, attn_row: torch.Tensor, attn_col: torch.Tensor,
                                  weight: torch.Tensor, bias: torch.Tensor, csr, csc,
                                  perm: torch.Tensor, negative_slope: float,
                                  attn_drop: float) -> torch.Tensor:
    """collapsed_gat_mean_bias_silu(attn_row, attn_col, ..., in_feat=lin(x).view(N,H,C), bias)
    evaluated aggregate-first: x [N,D] (16-byte aligned, D % 4 == 0), lin.weight
    [H*C, D] (C % 4 == 0), attn_row = alpha_dst and attn_col = alpha_src [N,H].
    Same dropout stream (call counter and keep bits) as the collapsed form."""
    if x.dtype != torch.float32 or x.device.type != "cuda" or x.dim() != 2:
        raise TypeError("aggregate-first GAT requires CUDA float32 x [N,D]")
    H = int(attn_row.size(1))
    if not (1 <= H <= MAX_HEADS):
        raise ValueError(f"collapsed GAT requires 1<=H<={MAX_HEADS}; got H={H}")
    if weight.dim() != 2 or weight.size(0) % H != 0 or weight.size(1) != x.size(1):
        raise ValueError("weight must be [H*C, D]")
    if not (0.0 <= float(attn_drop) < 1.0):
        raise ValueError("attn_drop must be in [0,1)")
    (rowptr, col), (row, colptr) = csr, csc
    plan = gat_plan_for(rowptr, col, row, colptr, perm)
    if plan.n_cols != x.size(0) or attn_row.size(0) != plan.n or attn_col.size(0) != plan.n_cols:
        raise RuntimeError(f"graph is {plan.n} x {plan.n_cols} but x has {x.size(0)} rows, "
                           f"attn_row {attn_row.size(0)}, attn_col {attn_col.size(0)}")
    seed = gat_call_seed(attn_drop)
    return aggregate_first_with_plan(x.contiguous(), attn_row.contiguous(), attn_col.contiguous(),
                                     weight, bias, plan, H, float(negative_slope),
                                     float(attn_drop), seed)


def collapsed_gat_aggregate_first_lin(x: torch.Tensor, attn_row: torch.Tensor,
                                      attn_col: torch.Tensor, weight: torch.Tensor, csr, csc,
                                      perm: torch.Tensor, negative_slope: float,
                                      attn_drop: float) -> torch.Tensor:
    """The head-mean output of collapsed_gat_aggregate_first before its bias and
    SiLU ([N, C]); pair it with gat_silu_add_layernorm.  Same arguments,
    checks and dropout stream."""
    if x.dtype != torch.float32 or x.device.type != "cuda" or x.dim() != 2:
        raise TypeError("aggregate-first GAT requires CUDA float32 x [N,D]")
    H = int(attn_row.size(1))
    if not (1 <= H <= MAX_HEADS):
        raise ValueError(f"collapsed GAT requires 1<=H<={MAX_HEADS}; got H={H}")
    if weight.dim() != 2 or weight.size(0) % H != 0 or weight.size(1) != x.size(1):
        raise ValueError("weight must be [H*C, D]")
    if not (0.0 <= float(attn_drop) < 1.0):
        raise ValueError("attn_drop must be in [0,1)")
    (rowptr, col), (row, colptr) = csr, csc
    plan = gat_plan_for(rowptr, col, row, colptr, perm)
    if plan.n_cols != x.size(0) or attn_row.size(0) != plan.n or attn_col.size(0) != plan.n_cols:
        raise RuntimeError(f"graph is {plan.n} x {plan.n_cols} but x has {x.size(0)} rows, "
                           f"attn_row {attn_row.size(0)}, attn_col {attn_col.size(0)}")
    seed = gat_call_seed(attn_drop)
    return _AggregateFirstLinFn.apply(x.contiguous(), attn_row.contiguous(),
                                      attn_col.contiguous(), weight, plan, H,
                                      float(negative_slope), float(attn_drop), seed)
