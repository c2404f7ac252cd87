"""Block side ops (drop-in for the reference's fused_block_ops,
fused_block_ops.py:1-121):

* ``fused_dropout_layernorm(x, weight, bias, dropout_p, eps)``
* ``fused_add_layernorm(a, b, weight, bias, eps)``
* ``fused_dropout_gamma_residual(h, g, gamma, dropout_p)`` = h + gamma*dropout(g)
* ``ensure_fused_block_ops_loaded(verbose=False)``

Dropout streams match the reference bit for bit: the per-call seed is
``(initial_seed & (2^63-1)) + 0x9E3779B97F4A7C15*call + 0xD2B74407B1CE6E93*tag``
modulo 2^63 with one module-level counter shared by both dropout ops
(tag 1 = dropout-LN, tag 2 = gamma residual; p == 0 gives seed 0 and does not
advance the counter, fused_block_ops.py:46-50), and element idx = n*D + d is
kept iff its 53-bit splitmix64 uniform is >= p.  Masks are recomputed in
backward from the seed.  Any D with D <= 1024 (D % 4 == 0) or D <= 256 runs
natively; the reference's generic kernels stop at D = 256 (:104).
"""
from __future__ import annotations

import torch

from . import _lib, seeds

_EXT = None
_EXT_ERROR = None
_CALL_COUNTER = seeds.counter_iter(seeds.BLOCK)  # block-op call ids (shared with seeds.next_seed)
MAX_D = 1024


def _extension_name():
    return "cign_sm100_block_ops"


def ensure_fused_block_ops_loaded(verbose: bool = False):
    global _EXT, _EXT_ERROR
    if _EXT is not None:
        return _EXT
    if _EXT_ERROR is not None:
        raise RuntimeError("block-op extension previously failed to load") from _EXT_ERROR
    if not torch.cuda.is_available():
        raise RuntimeError("Generalized fused block ops require CUDA")
    try:
        _EXT = _lib.load_library()
    except Exception as exc:
        _EXT_ERROR = exc
        raise
    return _EXT


def _next_seed(tag: int, dropout_p: float):
    """Seed of the next block-op call: an int, or a device seed slot while a
    seeds.DeviceSeedTable records."""
    return seeds.next_seed(seeds.BLOCK, dropout_p, tag)


# ------------------------------------------------------------------ raw ops
def dropout_ln_forward(x, w, b, p, eps, seed):
    lib = ensure_fused_block_ops_loaded()
    n, D = (int(s) for s in x.shape)
    y = torch.empty_like(x)
    mean = torch.empty((n,), dtype=torch.float32, device=x.device)
    rstd = torch.empty_like(mean)
    with _lib.DeviceGuard(x.device):
        rc = lib.cign_dropout_ln_fwd(n, D, _lib.ptr(x), _lib.ptr(w), _lib.ptr(b), float(p), float(eps),
                                     *_lib.seed_args(seed), _lib.ptr(y), _lib.ptr(mean),
                                     _lib.ptr(rstd), _lib.stream_of(x))
    _lib.check(rc, "cign_dropout_ln_fwd")
    return y, mean, rstd


def dropout_ln_backward(gy, x, w, mean, rstd, p, seed, addend=None):
    """(grad_x, grad_w, grad_b); with addend ([N, D], x's gradient from another
    consumer) grad_x includes it (cign_dropout_ln_bwd_add, no separate add)."""
    lib = ensure_fused_block_ops_loaded()
    n, D = (int(s) for s in x.shape)
    gx = torch.empty_like(x)
    gw = torch.empty((D,), dtype=torch.float32, device=x.device)
    gb = torch.empty_like(gw)
    ws = _lib.workspace(lib.cign_ln_bwd_workspace_bytes(n, D), x.device)
    with _lib.DeviceGuard(x.device):
        if addend is None:
            rc = lib.cign_dropout_ln_bwd(n, D, _lib.ptr(gy), _lib.ptr(x), _lib.ptr(w),
                                         _lib.ptr(mean), _lib.ptr(rstd), float(p),
                                         *_lib.seed_args(seed), _lib.ptr(gx), _lib.ptr(gw),
                                         _lib.ptr(gb), _lib.ptr(ws), ws.numel(), _lib.stream_of(x))
            name = "cign_dropout_ln_bwd"
        else:
            addend = addend.contiguous()
            if addend.shape != x.shape or addend.dtype != torch.float32:
                raise ValueError("addend must be a float32 tensor shaped like x")
            rc = lib.cign_dropout_ln_bwd_add(n, D, _lib.ptr(gy), _lib.ptr(x), _lib.ptr(w),
                                             _lib.ptr(mean), _lib.ptr(rstd), float(p),
                                             *_lib.seed_args(seed), _lib.ptr(addend),
                                             _lib.ptr(gx), _lib.ptr(gw), _lib.ptr(gb),
                                             _lib.ptr(ws), ws.numel(), _lib.stream_of(x))
            name = "cign_dropout_ln_bwd_add"
    _lib.check(rc, name)
    return gx, gw, gb


def add_ln_forward(a, b, w, bias, eps):
    lib = ensure_fused_block_ops_loaded()
    n, D = (int(s) for s in a.shape)
    y = torch.empty_like(a)
    mean = torch.empty((n,), dtype=torch.float32, device=a.device)
    rstd = torch.empty_like(mean)
    with _lib.DeviceGuard(a.device):
        rc = lib.cign_add_ln_fwd(n, D, _lib.ptr(a), _lib.ptr(b), _lib.ptr(w), _lib.ptr(bias),
                                 float(eps), _lib.ptr(y), _lib.ptr(mean), _lib.ptr(rstd),
                                 _lib.stream_of(a))
    _lib.check(rc, "cign_add_ln_fwd")
    return y, mean, rstd


def add_ln_backward(gy, a, b, w, mean, rstd):
    lib = ensure_fused_block_ops_loaded()
    n, D = (int(s) for s in a.shape)
    gz = torch.empty_like(a)
    gw = torch.empty((D,), dtype=torch.float32, device=a.device)
    gb = torch.empty_like(gw)
    ws = _lib.workspace(lib.cign_ln_bwd_workspace_bytes(n, D), a.device)
    with _lib.DeviceGuard(a.device):
        rc = lib.cign_add_ln_bwd(n, D, _lib.ptr(gy), _lib.ptr(a), _lib.ptr(b), _lib.ptr(w),
                                 _lib.ptr(mean), _lib.ptr(rstd), _lib.ptr(gz), _lib.ptr(gw),
                                 _lib.ptr(gb), _lib.ptr(ws), ws.numel(), _lib.stream_of(a))
    _lib.check(rc, "cign_add_ln_bwd")
    return gz, gw, gb


def gamma_residual_forward(h, g, gamma, p, seed):
    lib = ensure_fused_block_ops_loaded()
    n, D = (int(s) for s in h.shape)
    y = torch.empty_like(h)
    with _lib.DeviceGuard(h.device):
        rc = lib.cign_gamma_residual_fwd(n, D, _lib.ptr(h), _lib.ptr(g), _lib.ptr(gamma), float(p),
                                         *_lib.seed_args(seed), _lib.ptr(y), _lib.stream_of(h))
    _lib.check(rc, "cign_gamma_residual_fwd")
    return y


def gamma_residual_backward(gy, g, gamma, p, seed):
    lib = ensure_fused_block_ops_loaded()
    n, D = (int(s) for s in g.shape)
    gg = torch.empty_like(g)
    ggamma = torch.empty((D,), dtype=torch.float32, device=g.device)
    ws = _lib.workspace(lib.cign_gamma_residual_bwd_workspace_bytes(n, D), g.device)
    with _lib.DeviceGuard(g.device):
        rc = lib.cign_gamma_residual_bwd(n, D, _lib.ptr(gy), _lib.ptr(g), _lib.ptr(gamma), float(p),
                                         *_lib.seed_args(seed), _lib.ptr(gg), _lib.ptr(ggamma),
                                         _lib.ptr(ws), ws.numel(), _lib.stream_of(g))
    _lib.check(rc, "cign_gamma_residual_bwd")
    return gg, ggamma


def block_dropout_mask(count: int, p: float, seed: int, device) -> torch.Tensor:
    """uint8 keep-mask for element indices 0..count-1 (parity checks only)."""
    lib = ensure_fused_block_ops_loaded()
    mask = torch.empty((int(count),), dtype=torch.uint8, device=device)
    with _lib.DeviceGuard(device):
        rc = lib.cign_block_dropout_mask(int(count), float(p), *_lib.seed_args(seed),
                                         _lib.ptr(mask), _lib.stream_on(device))
    _lib.check(rc, "cign_block_dropout_mask")
    return mask


# ------------------------------------------------------------------ autograd
class _DropoutLayerNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, dropout_p, eps, seed):
        x = x.contiguous()
        weight = weight.contiguous()
        y, mean, rstd = dropout_ln_forward(x, weight, bias.contiguous(), dropout_p, eps, seed)
        ctx.save_for_backward(x, weight, mean, rstd)
        ctx.dropout_p = float(dropout_p)
        ctx.seed = seed
        return y

    @staticmethod
    def backward(ctx, grad_y):
        x, weight, mean, rstd = ctx.saved_tensors
        gx, gw, gb = dropout_ln_backward(grad_y.to(torch.float32).contiguous(), x, weight, mean, rstd,
                                         ctx.dropout_p, ctx.seed)
        return gx, gw, gb, None, None, None


class _AddLayerNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b, weight, bias, eps):
        a = a.contiguous()
        b = b.contiguous()
        weight = weight.contiguous()
        y, mean, rstd = add_ln_forward(a, b, weight, bias.contiguous(), eps)
        ctx.save_for_backward(a, b, weight, mean, rstd)
        return y

    @staticmethod
    def backward(ctx, grad_y):
        a, b, weight, mean, rstd = ctx.saved_tensors
        gz, gw, gb = add_ln_backward(grad_y.to(torch.float32).contiguous(), a, b, weight, mean, rstd)
        return gz, gz, gw, gb, None


class _DropoutGammaResidualFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, g, gamma, dropout_p, seed):
        g = g.contiguous()
        gamma = gamma.contiguous()
        y = gamma_residual_forward(h.contiguous(), g, gamma, dropout_p, seed)
        ctx.save_for_backward(g, gamma)
        ctx.dropout_p = float(dropout_p)
        ctx.seed = seed
        return y

    @staticmethod
    def backward(ctx, grad_y):
        g, gamma = ctx.saved_tensors
        grad_y = grad_y.to(torch.float32).contiguous()
        gg, ggamma = gamma_residual_backward(grad_y, g, gamma, ctx.dropout_p, ctx.seed)
        return grad_y, gg, ggamma, None, None


def _check_2d(x, name):
    if x.device.type != "cuda" or x.dtype != torch.float32:
        raise TypeError(f"{name} must be CUDA float32")
    if x.dim() != 2 or not (1 <= x.size(1) <= MAX_D):
        raise ValueError(f"{name} must be [N,D] with 1<=D<={MAX_D}, got {tuple(x.shape)}")
    return int(x.size(1))


def fused_dropout_layernorm(x, weight, bias, dropout_p, eps):
    D = _check_2d(x, "x")
    if weight.numel() != D or bias.numel() != D:
        raise ValueError("LayerNorm weight/bias must match hidden dimension")
    if not (0.0 <= float(dropout_p) < 1.0):
        raise ValueError("dropout_p must be in [0,1)")
    return _DropoutLayerNormFn.apply(x, weight, bias, float(dropout_p), float(eps),
                                     _next_seed(1, dropout_p))


def fused_add_layernorm(a, b, weight, bias, eps):
    D = _check_2d(a, "a")
    _check_2d(b, "b")
    if a.shape != b.shape or weight.numel() != D or bias.numel() != D:
        raise ValueError("Add+LayerNorm shapes do not match")
    return _AddLayerNormFn.apply(a, b, weight, bias, float(eps))


def fused_dropout_gamma_residual(h, g, gamma, dropout_p):
    D = _check_2d(h, "h")
    _check_2d(g, "g")
    if h.shape != g.shape:
        raise ValueError("h and g must have the same shape")
    if gamma.dim() != 1 or gamma.numel() != D:
        raise ValueError(f"vector gamma must have shape [{D}]")
    if not (0.0 <= float(dropout_p) < 1.0):
        raise ValueError("dropout_p must be in [0,1)")
    return _DropoutGammaResidualFn.apply(h, g, gamma, float(dropout_p), _next_seed(2, dropout_p))
