"""Fixed-CSR k-hop propagation on sm_100a (drop-in for the reference module).

Same public names, signatures and autograd semantics as the reference's
``multihop_csr_pipeline`` (multihop_csr_pipeline.py:1-350):

* ``ensure_multihop_csr_loaded()``
* ``MultiHopCSR3GraphOperator(base_fixed_csr, dense_cols, algorithm=2)`` with
  ``.plan.{prepare, forward3, backward3, workspace_bytes, info, algorithm}``
* ``HybridNative3TailCSRGraphOperator`` / ``hybrid_native3_tail_csr``
* ``GenericMultiHopCSRGraphOperator`` / ``generic_multihop_csr``
* ``prepare_multihop_csr_operator(base, dense_cols, algorithm=2,
  powers=(1, 2, 3), prefer_native_three_hop=True, strategy="auto")``
* ``multihop_csr3(op, x) -> (y1, y2, y3)``

All three operator kinds run the same native k-hop kernels
(``cign_multihop_fwd`` / ``cign_multihop_bwd``): the reference's split into a
cuSPARSE 3-hop prefix plus a torch tail (and its pure-torch generic path)
collapses into one path.  ``algorithm`` is accepted and validated for API
compatibility (it selected a cuSPARSE SpMM algorithm) and reported in
``info``; it does not change the computation.
"""
from __future__ import annotations

from typing import Dict, Tuple

import torch

from . import _lib
from .plans import SpmmPlan

_EXT = None


def ensure_multihop_csr_loaded():
    """Load the native library once (multihop_csr_pipeline.py:15-35)."""
    global _EXT
    if _EXT is not None:
        return _EXT
    if not torch.cuda.is_available():
        raise RuntimeError("A3-v5 MultiHopCSR requires CUDA.")
    _EXT = _lib.load_library()
    return _EXT


def _csr_parts_int32(csr: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """int32 clones of a CUDA fp32 CSR (multihop_csr_pipeline.py:38-48)."""
    if csr.layout != torch.sparse_csr:
        raise TypeError(f"Expected sparse CSR tensor, got {csr.layout}.")
    if csr.device.type != "cuda":
        raise RuntimeError("A3-v5 CSR tensors must already be on CUDA.")
    if csr.dtype != torch.float32:
        raise TypeError(f"A3-v5 currently requires float32 sparse values, got {csr.dtype}.")
    crow = csr.crow_indices().to(dtype=torch.int32).clone().contiguous()
    col = csr.col_indices().to(dtype=torch.int32).clone().contiguous()
    val = csr.values().to(dtype=torch.float32).clone().contiguous()
    return crow, col, val


class _NativePlan:
    """The ``.plan`` object of the reference's MultiHopCsrPlan, backed by
    a ``cign_spmm_plan`` (multihop_csr_ext/multihop_csr_pipeline_cuda.cu:113-322)."""

    def __init__(self, p, pt, rows: int, dense_cols: int, algorithm: int):
        self.spmm = SpmmPlan(p[0], p[1], p[2], pt[0], pt[1], pt[2])
        self.rows = int(rows)
        self.dense_cols = int(dense_cols)
        self.algorithm = int(algorithm)

    def prepare(self, dummy: torch.Tensor) -> None:
        if dummy.dim() != 2 or dummy.size(0) != self.rows:
            raise RuntimeError("prepare: dense operand must be [rows, dense_cols]")

    def workspace_bytes(self) -> int:
        # One [rows, F] fp32 ping-pong buffer for the backward chain; it is
        # allocated per call from torch's caching allocator.
        return self.rows * self.dense_cols * 4

    def info(self) -> Dict[str, object]:
        d = dict(self.spmm.info())
        d["symmetric_operator"] = bool(self.spmm.symmetric)
        return d

    def forward3(self, x: torch.Tensor):
        return tuple(self.spmm.forward(x, 3))

    def backward3(self, g1, g2, g3):
        return self.spmm.backward([g1, g2, g3], int(g1.size(1)))


def _powers_info(powers):
    pset = tuple(sorted(set(int(p) for p in powers)))
    if not pset or min(pset) < 0:
        raise ValueError(f"powers must be non-empty non-negative integers, got {pset}")
    positive = tuple(p for p in pset if p > 0)
    return pset, positive, (max(positive) if positive else 0)


class _MultiHopFunction(torch.autograd.Function):
    """Y_p = P^p x for the requested positive powers; backward
    acc = P^T (acc + g_p) from the top power down
    (multihop_csr_pipeline.py:59-86 and :233-265)."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, plan: SpmmPlan, positive_powers, max_power: int):
        ctx.input_dtype = x.dtype
        ctx.plan = plan
        ctx.positive_powers = tuple(positive_powers)
        ctx.max_power = int(max_power)
        x32 = x.to(dtype=torch.float32).contiguous()
        ctx.F = int(x32.size(1))
        ys = plan.forward(x32, ctx.max_power)
        return tuple(ys[p - 1] for p in ctx.positive_powers)

    @staticmethod
    def backward(ctx, *grad_outputs):
        if all(g is None for g in grad_outputs):
            return None, None, None, None
        grads = [None] * ctx.max_power
        for p, g in zip(ctx.positive_powers, grad_outputs):
            if g is not None:
                grads[p - 1] = g.to(dtype=torch.float32).contiguous()
        gx = ctx.plan.backward(grads, ctx.F)
        if gx.dtype != ctx.input_dtype:
            gx = gx.to(ctx.input_dtype)
        return gx, None, None, None


class MultiHopCSR3Function(torch.autograd.Function):
    """Reference name kept (multihop_csr_pipeline.py:59-86): the 3-hop case."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, operator: "MultiHopCSR3GraphOperator"):
        ctx.input_dtype = x.dtype
        ctx.operator = operator
        x32 = x.to(dtype=torch.float32).contiguous()
        y1, y2, y3 = operator.plan.forward3(x32)
        return y1, y2, y3

    @staticmethod
    def backward(ctx, grad_y1, grad_y2, grad_y3):
        ref = grad_y1 if grad_y1 is not None else (grad_y2 if grad_y2 is not None else grad_y3)
        if ref is None:
            return None, None
        gs = [None if g is None else g.to(dtype=torch.float32).contiguous()
              for g in (grad_y1, grad_y2, grad_y3)]
        grad_x = ctx.operator.plan.spmm.backward(gs, int(ref.size(1)))
        if grad_x.dtype != ctx.input_dtype:
            grad_x = grad_x.to(ctx.input_dtype)
        return grad_x, None


class MultiHopCSR3GraphOperator:
    __slots__ = (
        "base", "plan", "_storage_p", "_storage_pt", "shape", "nnz", "dtype",
        "device", "dense_cols", "algorithm", "powers", "info",
    )

    def __init__(self, base_fixed_csr, dense_cols: int, algorithm: int = 2):
        if int(dense_cols) <= 0:
            raise ValueError("dense_cols must be positive.")
        if int(algorithm) not in (1, 2, 3):
            raise ValueError("A3-v5 cuSPARSE algorithm must be 1, 2, or 3.")
        if not hasattr(base_fixed_csr, "csr") or not hasattr(base_fixed_csr, "csr_t"):
            raise TypeError("A3-v5 expects an already prepared FixedCSRGraphOperator.")
        self.base = base_fixed_csr
        self.shape = tuple(base_fixed_csr.shape)
        self.nnz = int(base_fixed_csr.nnz)
        self.dtype = base_fixed_csr.dtype
        self.device = base_fixed_csr.device
        self.dense_cols = int(dense_cols)
        self.algorithm = int(algorithm)
        self.powers = (1, 2, 3)
        p = _csr_parts_int32(base_fixed_csr.csr)
        pt = _csr_parts_int32(base_fixed_csr.csr_t)
        self._storage_p = p
        self._storage_pt = pt
        ensure_multihop_csr_loaded()
        self.plan = _NativePlan(p, pt, int(self.shape[0]), self.dense_cols, self.algorithm)
        dummy = torch.empty((self.shape[0], self.dense_cols), device=self.device, dtype=torch.float32)
        self.plan.prepare(dummy)
        torch.cuda.synchronize(self.device)
        self.info: Dict[str, object] = {
            "backend": "cign_sm100_multihop",
            "powers": list(self.powers),
            "shape": self.shape,
            "nnz": self.nnz,
            "dense_cols": self.dense_cols,
            "index_dtype": "torch.int32",
            "algorithm": self.algorithm,
            "workspace_bytes": int(self.plan.workspace_bytes()),
            "native_info": self.plan.info(),
        }

    @property
    def csr(self):
        return self.base.csr

    @property
    def csr_t(self):
        return self.base.csr_t


class HybridNative3TailCSRGraphOperator:
    """Arbitrary-K propagation (multihop_csr_pipeline.py:160-211); here the
    whole recurrence is native (no torch tail)."""

    __slots__ = (
        "base", "native3", "shape", "nnz", "dtype", "device", "dense_cols",
        "algorithm", "powers", "positive_powers", "max_power", "info",
    )

    def __init__(self, base_fixed_csr, dense_cols: int, powers, algorithm: int = 2):
        powers, positive, max_power = _powers_info(powers)
        if not positive or max(positive) < 3:
            raise ValueError(
                "HybridNative3TailCSR requires at least one positive requested power >= 3; "
                f"got powers={powers}"
            )
        self.base = base_fixed_csr
        self.native3 = MultiHopCSR3GraphOperator(base_fixed_csr, dense_cols=dense_cols, algorithm=algorithm)
        self.shape = tuple(base_fixed_csr.shape)
        self.nnz = int(base_fixed_csr.nnz)
        self.dtype = base_fixed_csr.dtype
        self.device = base_fixed_csr.device
        self.dense_cols = int(dense_cols)
        self.algorithm = int(algorithm)
        self.powers = powers
        self.positive_powers = positive
        self.max_power = max_power
        self.info = {
            "backend": "cign_sm100_multihop",
            "powers": list(self.powers),
            "shape": self.shape,
            "nnz": self.nnz,
            "dense_cols": self.dense_cols,
            "algorithm": self.algorithm,
            "implementation": "native k-hop recurrence (one launch per hop)",
            "native_info": self.native3.info,
        }

    @property
    def csr(self):
        return self.base.csr

    @property
    def csr_t(self):
        return self.base.csr_t


def hybrid_native3_tail_csr(operator: "HybridNative3TailCSRGraphOperator", x: torch.Tensor):
    """dict{power: P^power x} for the requested positive powers."""
    ys = _MultiHopFunction.apply(x, operator.native3.plan.spmm, operator.positive_powers,
                                 operator.max_power)
    return {p: y for p, y in zip(operator.positive_powers, ys)}


class GenericMultiHopCSRFunction(torch.autograd.Function):
    """Reference name kept (multihop_csr_pipeline.py:233-265)."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, operator: "GenericMultiHopCSRGraphOperator"):
        return _MultiHopFunction.forward(ctx, x, operator._plan().spmm, operator.positive_powers,
                                         operator.max_power)

    @staticmethod
    def backward(ctx, *grad_outputs):
        gx = _MultiHopFunction.backward(ctx, *grad_outputs)[0]
        return gx, None


class GenericMultiHopCSRGraphOperator:
    __slots__ = (
        "base", "shape", "nnz", "dtype", "device", "dense_cols", "algorithm",
        "powers", "positive_powers", "max_power", "info", "_native",
    )

    def __init__(self, base_fixed_csr, dense_cols: int, powers, algorithm: int = 2):
        if not hasattr(base_fixed_csr, "csr") or not hasattr(base_fixed_csr, "csr_t"):
            raise TypeError("GenericMultiHopCSR expects an already prepared FixedCSRGraphOperator.")
        powers, positive, max_power = _powers_info(powers)
        self.base = base_fixed_csr
        self.shape = tuple(base_fixed_csr.shape)
        self.nnz = int(base_fixed_csr.nnz)
        self.dtype = base_fixed_csr.dtype
        self.device = base_fixed_csr.device
        self.dense_cols = int(dense_cols)
        self.algorithm = int(algorithm)
        self.powers = powers
        self.positive_powers = positive
        self.max_power = max_power
        self._native = None
        self.info = {
            "backend": "cign_sm100_multihop",
            "powers": list(self.powers),
            "shape": self.shape,
            "nnz": self.nnz,
            "dense_cols": self.dense_cols,
            "value_dtype": str(self.dtype),
            "implementation": "native k-hop recurrence + single custom autograd node",
        }

    def _plan(self) -> _NativePlan:
        if self._native is None:
            p = _csr_parts_int32(self.base.csr)
            pt = _csr_parts_int32(self.base.csr_t)
            self._native = _NativePlan(p, pt, int(self.shape[0]), self.dense_cols, self.algorithm)
        return self._native

    @property
    def csr(self):
        return self.base.csr

    @property
    def csr_t(self):
        return self.base.csr_t


def prepare_multihop_csr_operator(
    base_fixed_csr,
    dense_cols: int,
    algorithm: int = 2,
    powers=(1, 2, 3),
    prefer_native_three_hop: bool = True,
    strategy: str = "auto",
):
    """Same selection rules and return types as multihop_csr_pipeline.py:309-337."""
    pset = tuple(sorted(set(int(p) for p in powers)))
    positive = tuple(p for p in pset if p > 0)
    max_power = max(positive) if positive else 0
    strategy = str(strategy).strip().lower()
    if strategy not in {"auto", "native3_tail", "generic"}:
        raise ValueError(f"Unknown MultiHop strategy={strategy!r}")
    if prefer_native_three_hop and pset == (1, 2, 3):
        return MultiHopCSR3GraphOperator(base_fixed_csr, dense_cols=dense_cols, algorithm=algorithm)
    if strategy in {"auto", "native3_tail"} and max_power >= 3:
        return HybridNative3TailCSRGraphOperator(base_fixed_csr, dense_cols=dense_cols, powers=pset,
                                                 algorithm=algorithm)
    op = GenericMultiHopCSRGraphOperator(base_fixed_csr, dense_cols=dense_cols, powers=pset,
                                         algorithm=algorithm)
    if positive:
        ensure_multihop_csr_loaded()
        op._plan()
    return op


def multihop_csr3(operator: MultiHopCSR3GraphOperator, x: torch.Tensor):
    return MultiHopCSR3Function.apply(x, operator)


def generic_multihop_csr(operator: GenericMultiHopCSRGraphOperator, x: torch.Tensor):
    if not operator.positive_powers:
        return {}
    vals = GenericMultiHopCSRFunction.apply(x, operator)
    if len(operator.positive_powers) == 1 and torch.is_tensor(vals):
        vals = (vals,)
    return {p: y for p, y in zip(operator.positive_powers, vals)}
