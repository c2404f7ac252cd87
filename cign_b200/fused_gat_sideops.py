"""GAT side ops (drop-in for the reference's fused_gat_sideops).

* ``fused_attention_logits(x, att_src, att_dst) -> (alpha_src, alpha_dst)``:
  ``alpha[n,h] = sum_c x[n,h,c] * att[0,h,c]`` with gradients for x and both
  attention vectors (fused_gat_sideops.py:50-97).
* ``fused_head_mean_bias_silu(out, bias) -> SiLU(mean_h out + bias)``
  (fused_gat_sideops.py:73-105).
* ``ensure_fused_gat_sideops_loaded(verbose=False)``.

Parameter gradients use a fixed two-stage reduction (deterministic).
"""
from __future__ import annotations

import torch

from . import _lib

_EXT = None
_EXT_ERROR = None


def _extension_name() -> str:
    return "cign_sm100_gat_sideops"


def ensure_fused_gat_sideops_loaded(verbose: bool = False):
    global _EXT, _EXT_ERROR
    if _EXT is not None:
        return _EXT
    if _EXT_ERROR is not None:
        raise RuntimeError("GAT side-op extension previously failed to load") from _EXT_ERROR
    if not torch.cuda.is_available():
        raise RuntimeError("A3-v3 fused GAT side ops require CUDA")
    try:
        _EXT = _lib.load_library()
    except Exception as exc:
        _EXT_ERROR = exc
        raise
    return _EXT


def attention_logits_forward(x, att_src, att_dst):
    lib = ensure_fused_gat_sideops_loaded()
    n, H, C = (int(s) for s in x.shape)
    if att_src.numel() != H * C or att_dst.numel() != H * C:
        raise RuntimeError("att_src/att_dst must have H*C elements")
    a_src = torch.empty((n, H), dtype=torch.float32, device=x.device)
    a_dst = torch.empty_like(a_src)
    with _lib.DeviceGuard(x.device):
        rc = lib.cign_attn_logits_fwd(n, H, C, _lib.ptr(x), _lib.ptr(att_src), _lib.ptr(att_dst),
                                      _lib.ptr(a_src), _lib.ptr(a_dst), _lib.stream_of(x))
    _lib.check(rc, "cign_attn_logits_fwd")
    return a_src, a_dst


def attention_logits_backward(grad_src, grad_dst, x, att_src, att_dst, grad_x=None):
    """Returns (grad_x, grad_att_src, grad_att_dst); adds into grad_x if given."""
    lib = ensure_fused_gat_sideops_loaded()
    n, H, C = (int(s) for s in x.shape)
    acc = grad_x is not None
    if grad_x is None:
        grad_x = torch.empty_like(x)
    g_as = torch.empty(att_src.shape, dtype=torch.float32, device=x.device)
    g_ad = torch.empty(att_dst.shape, dtype=torch.float32, device=x.device)
    ws = _lib.workspace(lib.cign_attn_logits_bwd_workspace_bytes(n, H, C), x.device)
    with _lib.DeviceGuard(x.device):
        rc = lib.cign_attn_logits_bwd(n, H, C, _lib.ptr(grad_src), _lib.ptr(grad_dst), _lib.ptr(x),
                                      _lib.ptr(att_src), _lib.ptr(att_dst), _lib.ptr(grad_x),
                                      _lib.ptr(g_as), _lib.ptr(g_ad), 1 if acc else 0,
                                      _lib.ptr(ws), ws.numel(), _lib.stream_of(x))
    _lib.check(rc, "cign_attn_logits_bwd")
    return grad_x, g_as, g_ad


class _AttentionLogitsFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, att_src, att_dst):
        x = x.contiguous()
        att_src = att_src.contiguous()
        att_dst = att_dst.contiguous()
        a_src, a_dst = attention_logits_forward(x, att_src, att_dst)
        ctx.save_for_backward(x, att_src, att_dst)
        return a_src, a_dst

    @staticmethod
    def backward(ctx, grad_src, grad_dst):
        x, att_src, att_dst = ctx.saved_tensors
        if grad_src is None:
            grad_src = torch.zeros(x.shape[:2], dtype=torch.float32, device=x.device)
        if grad_dst is None:
            grad_dst = torch.zeros(x.shape[:2], dtype=torch.float32, device=x.device)
        grad_x, g_as, g_ad = attention_logits_backward(
            grad_src.to(torch.float32).contiguous(), grad_dst.to(torch.float32).contiguous(), x,
            att_src, att_dst)
        return grad_x, g_as, g_ad


class _HeadMeanBiasSiLUFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, out, bias):
        lib = ensure_fused_gat_sideops_loaded()
        out = out.contiguous()
        bias = bias.contiguous()
        n, H, C = (int(s) for s in out.shape)
        y = torch.empty((n, C), dtype=torch.float32, device=out.device)
        pre = torch.empty_like(y)
        with _lib.DeviceGuard(out.device):
            rc = lib.cign_head_mean_bias_silu_fwd(n, H, C, _lib.ptr(out), _lib.ptr(bias), _lib.ptr(y),
                                                  _lib.ptr(pre), _lib.stream_of(out))
        _lib.check(rc, "cign_head_mean_bias_silu_fwd")
        ctx.save_for_backward(pre)
        ctx.heads = H
        return y

    @staticmethod
    def backward(ctx, grad_y):
        lib = ensure_fused_gat_sideops_loaded()
        (pre,) = ctx.saved_tensors
        grad_y = grad_y.to(torch.float32).contiguous()
        n, C = (int(s) for s in pre.shape)
        H = ctx.heads
        grad_out = torch.empty((n, H, C), dtype=torch.float32, device=pre.device)
        grad_bias = torch.empty((C,), dtype=torch.float32, device=pre.device)
        ws = _lib.workspace(lib.cign_head_mean_bias_silu_bwd_workspace_bytes(n, C), pre.device)
        with _lib.DeviceGuard(pre.device):
            rc = lib.cign_head_mean_bias_silu_bwd(n, H, C, _lib.ptr(grad_y), _lib.ptr(pre),
                                                  _lib.ptr(grad_out), _lib.ptr(grad_bias),
                                                  _lib.ptr(ws), ws.numel(), _lib.stream_of(pre))
        _lib.check(rc, "cign_head_mean_bias_silu_bwd")
        return grad_out, grad_bias


def fused_attention_logits(x: torch.Tensor, att_src: torch.Tensor, att_dst: torch.Tensor):
    if x.dtype != torch.float32 or x.device.type != "cuda":
        raise TypeError("A3-v3 fused attention logits require CUDA float32 tensors")
    return _AttentionLogitsFn.apply(x, att_src, att_dst)


def fused_head_mean_bias_silu(out: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    if bias is None:
        raise ValueError("A3-v3 fused head reduction currently requires GAT bias=True")
    if out.dtype != torch.float32 or out.device.type != "cuda":
        raise TypeError("A3-v3 fused head reduction requires CUDA float32 tensors")
    return _HeadMeanBiasSiLUFn.apply(out, bias)
