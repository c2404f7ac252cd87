"""Python owners of the native plan objects (cign_spmm_plan, cign_gat_plan).

A plan keeps the int32 CSR tensors it was built from alive (the native plan
only stores their device pointers) and is immutable after construction, so
one plan may serve several streams.  Plans are built once per graph, before
any timed work (the reference does the same in MultiHopCSR3GraphOperator /
prepare_fused_gat_graph).
"""
from __future__ import annotations

import ctypes
from collections import OrderedDict
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from . import _lib


def _as_i32(t: torch.Tensor) -> torch.Tensor:
    return t.to(dtype=torch.int32).contiguous()


class HopTimer:
    """Opt-in device timing of the k-hop calls: CUDA events recorded on the
    launching stream around every cign_multihop_fwd / _bwd call while the
    timer is installed (``SpmmPlan.hop_timer = HopTimer()``).  ``records`` holds
    (kind, n_hops, n_addend_hops, F, start, end); read them after a
    synchronize.  Inside a CUDA-graph capture the events become event-record
    nodes of the graph, so after a replay they hold that replay's times."""

    def __init__(self):
        self.records = []

    @staticmethod
    def _event(stream):
        ev = torch.cuda.Event(enable_timing=True,
                              external=torch.cuda.is_current_stream_capturing())
        ev.record(stream)
        return ev

    def begin(self, stream):
        return self._event(stream)

    def end(self, stream, start, kind, n_hops, n_addend, F, rows=None, nnz=None):
        self.records.append((kind, n_hops, n_addend, F, start, self._event(stream), rows, nnz))


class SpmmPlan:
    """Native SpMM plan over a square fixed operator P (and optionally P^T).

    ``crow/col/val`` (and the ``*_t`` triple) are int32/int32/fp32 CUDA
    tensors; when the transpose triple is None or bitwise equal to P's, the
    transposed products reuse P (symmetric operator, the default for CIGN's
    undirected normalised adjacency).
    """

    hop_timer: Optional[HopTimer] = None

    def __init__(self, crow, col, val, crow_t=None, col_t=None, val_t=None,
                 cols: Optional[int] = None):
        _lib.require_cuda("SpmmPlan")
        self.lib = _lib.load_library()
        self.device = crow.device
        self.crow, self.col, self.val = _as_i32(crow), _as_i32(col), val.to(torch.float32).contiguous()
        self.rows = int(self.crow.numel() - 1)
        self.cols = self.rows if cols is None else int(cols)
        self.nnz = int(self.col.numel())
        if self.cols != self.rows and crow_t is None:
            raise ValueError("a rectangular operator needs its transpose (crow_t, col_t, val_t)")
        symmetric = crow_t is None
        if not symmetric and self.cols == self.rows:
            crow_t, col_t = _as_i32(crow_t), _as_i32(col_t)
            val_t = val_t.to(torch.float32).contiguous()
            symmetric = (
                crow_t.numel() == self.crow.numel()
                and col_t.numel() == self.col.numel()
                and bool(torch.equal(crow_t, self.crow))
                and bool(torch.equal(col_t, self.col))
                and bool(torch.equal(val_t, self.val))
            )
        elif not symmetric:
            crow_t, col_t = _as_i32(crow_t), _as_i32(col_t)
            val_t = val_t.to(torch.float32).contiguous()
        self.symmetric = symmetric
        if symmetric:
            self.crow_t, self.col_t, self.val_t = self.crow, self.col, self.val
        else:
            self.crow_t, self.col_t, self.val_t = crow_t, col_t, val_t
        p = _lib.CsrF32(self.rows, self.cols, self.nnz, self.crow.data_ptr(), self.col.data_ptr(),
                        self.val.data_ptr())
        handle = ctypes.c_void_p()
        with _lib.DeviceGuard(self.device):
            if symmetric:
                rc = self.lib.cign_spmm_plan_create(ctypes.byref(p), None, ctypes.byref(handle))
            else:
                pt = _lib.CsrF32(self.cols, self.rows, int(self.col_t.numel()), self.crow_t.data_ptr(),
                                 self.col_t.data_ptr(), self.val_t.data_ptr())
                rc = self.lib.cign_spmm_plan_create(ctypes.byref(p), ctypes.byref(pt),
                                                    ctypes.byref(handle))
        _lib.check(rc, "cign_spmm_plan_create")
        self.handle = handle

    def __del__(self):
        h = getattr(self, "handle", None)
        if h is not None and h.value:
            try:
                self.lib.cign_spmm_plan_destroy(h)
            except Exception:
                pass
            self.handle = None

    def info(self) -> Dict[str, int]:
        inf = _lib.SpmmPlanInfo()
        _lib.check(self.lib.cign_spmm_plan_get_info(self.handle, ctypes.byref(inf)),
                   "cign_spmm_plan_get_info")
        return {name: int(getattr(inf, name)) for name, _ in _lib.SpmmPlanInfo._fields_}

    # ---------------------------------------------------------------- ops
    def _check_dense(self, x: torch.Tensor, what: str, rows: Optional[int] = None) -> torch.Tensor:
        rows = self.rows if rows is None else int(rows)
        if x.device != self.device:
            raise RuntimeError(f"{what}: tensor on {x.device}, plan on {self.device}")
        if x.dim() != 2 or x.size(0) != rows:
            raise ValueError(f"{what}: expected [{rows}, F], got {tuple(x.shape)}")
        return x.to(torch.float32).contiguous()

    def spmm(self, x: torch.Tensor, transpose: bool = False,
             addend: Optional[torch.Tensor] = None) -> torch.Tensor:
        x = self._check_dense(x, "spmm", self.rows if transpose else self.cols)
        F = int(x.size(1))
        y = torch.empty((self.cols if transpose else self.rows, F), dtype=torch.float32,
                        device=x.device)
        if addend is not None:
            addend = self._check_dense(addend, "spmm addend", int(y.size(0)))
        ws = _lib.workspace(self.lib.cign_spmm_workspace_bytes(self.handle, F), self.device)
        timer = SpmmPlan.hop_timer
        with _lib.DeviceGuard(self.device):
            t0 = timer.begin(torch.cuda.current_stream(self.device)) if timer else None
            rc = self.lib.cign_spmm(self.handle, 1 if transpose else 0, _lib.ptr(x), F,
                                    _lib.ptr(addend), _lib.ptr(y), _lib.ptr(ws), ws.numel(),
                                    _lib.stream_of(x))
            if timer:
                timer.end(torch.cuda.current_stream(self.device), t0, "bwd" if transpose else "fwd",
                          1, 0 if addend is None else 1, F, rows=int(y.size(0)), nnz=self.nnz)
        _lib.check(rc, "cign_spmm")
        return y

    def forward(self, x: torch.Tensor, max_power: int) -> List[torch.Tensor]:
        """[P^1 x, ..., P^max_power x]."""
        x = self._check_dense(x, "multihop forward")
        ys = [torch.empty_like(x) for _ in range(int(max_power))]
        arr = _lib.ptr_array(ys)
        F = int(x.size(1))
        ws = _lib.workspace(self.lib.cign_spmm_workspace_bytes(self.handle, F), self.device)
        timer = SpmmPlan.hop_timer
        with _lib.DeviceGuard(self.device):
            stream = _lib.stream_of(x)
            t0 = timer.begin(torch.cuda.current_stream(self.device)) if timer else None
            rc = self.lib.cign_multihop_fwd(self.handle, int(max_power), _lib.ptr(x), F, arr,
                                            _lib.ptr(ws), ws.numel(), stream)
            if timer:
                timer.end(torch.cuda.current_stream(self.device), t0, "fwd", int(max_power), 0, F)
        _lib.check(rc, "cign_multihop_fwd")
        return ys

    def forward_split(self, x0: torch.Tensor, x1: torch.Tensor,
                      max_power: int) -> List[torch.Tensor]:
        """forward(torch.cat([x0, x1], 1), max_power) without forming the
        concatenation: hop 1 reads the two [rows, d] blocks directly
        (cign_multihop_fwd_split; d % 256 == 0)."""
        x0 = self._check_dense(x0, "multihop forward (first block)")
        x1 = self._check_dense(x1, "multihop forward (second block)")
        d = int(x0.size(1))
        if x1.shape != x0.shape:
            raise ValueError("forward_split: the two column blocks must have the same shape")
        ys = [torch.empty((self.rows, 2 * d), dtype=torch.float32, device=self.device)
              for _ in range(int(max_power))]
        ws = _lib.workspace(self.lib.cign_spmm_workspace_bytes(self.handle, 2 * d), self.device)
        timer = SpmmPlan.hop_timer
        with _lib.DeviceGuard(self.device):
            t0 = timer.begin(torch.cuda.current_stream(self.device)) if timer else None
            rc = self.lib.cign_multihop_fwd_split(self.handle, int(max_power), _lib.ptr(x0),
                                                  _lib.ptr(x1), d, _lib.ptr_array(ys),
                                                  _lib.ptr(ws), ws.numel(), _lib.stream_of(x0))
            if timer:
                timer.end(torch.cuda.current_stream(self.device), t0, "fwd", int(max_power), 0,
                          2 * d)
        _lib.check(rc, "cign_multihop_fwd_split")
        return ys

    def spmm_bf16(self, x: torch.Tensor, out_dtype=torch.bfloat16,
                  transpose: bool = False) -> torch.Tensor:
        """P x (or P^T x) for bf16-stored features: fp32 accumulation, output
        fp32 or rounded to bf16 (cign_spmm_bf16); F % 8 == 0."""
        if x.dtype != torch.bfloat16:
            raise TypeError("spmm_bf16 needs a bfloat16 x")
        if out_dtype not in (torch.bfloat16, torch.float32):
            raise TypeError("out_dtype must be bfloat16 or float32")
        rows_in = self.rows if transpose else self.cols
        if x.device != self.device or x.dim() != 2 or x.size(0) != rows_in:
            raise ValueError(f"spmm_bf16: expected [{rows_in}, F] on {self.device}")
        x = x.contiguous()
        F = int(x.size(1))
        y = torch.empty((self.cols if transpose else self.rows, F), dtype=out_dtype,
                        device=x.device)
        ws = _lib.workspace(self.lib.cign_spmm_workspace_bytes(self.handle, F), self.device)
        with _lib.DeviceGuard(self.device):
            rc = self.lib.cign_spmm_bf16(self.handle, 1 if transpose else 0, _lib.ptr(x), F,
                                         _lib.ptr(y), 1 if out_dtype == torch.bfloat16 else 0,
                                         _lib.ptr(ws), ws.numel(), _lib.stream_of(x))
        _lib.check(rc, "cign_spmm_bf16")
        return y

    def forward_bf16(self, x: torch.Tensor, max_power: int) -> List[torch.Tensor]:
        """[P^1 x, ..., P^max_power x] with every hop stored as bf16 (fp32
        accumulation inside each hop; cign_multihop_fwd_bf16)."""
        if x.dtype != torch.bfloat16:
            raise TypeError("forward_bf16 needs a bfloat16 x")
        if x.device != self.device or x.dim() != 2 or x.size(0) != self.rows:
            raise ValueError(f"forward_bf16: expected [{self.rows}, F] on {self.device}")
        x = x.contiguous()
        ys = [torch.empty_like(x) for _ in range(int(max_power))]
        F = int(x.size(1))
        ws = _lib.workspace(self.lib.cign_spmm_workspace_bytes(self.handle, F), self.device)
        with _lib.DeviceGuard(self.device):
            rc = self.lib.cign_multihop_fwd_bf16(self.handle, int(max_power), _lib.ptr(x), F,
                                                 _lib.ptr_array(ys), _lib.ptr(ws), ws.numel(),
                                                 _lib.stream_of(x))
        _lib.check(rc, "cign_multihop_fwd_bf16")
        return ys

    def backward(self, grads: Sequence[Optional[torch.Tensor]], F: int) -> torch.Tensor:
        """grads[p-1] = dL/d(P^p x) or None; returns dL/dx."""
        ref = next((g for g in grads if g is not None), None)
        if ref is None:
            raise ValueError("multihop backward needs at least one gradient")
        gs = [None if g is None else self._check_dense(g, "multihop grad") for g in grads]
        gx = torch.empty((self.rows, int(F)), dtype=torch.float32, device=self.device)
        ws = _lib.workspace(self.lib.cign_multihop_workspace_bytes(self.handle, len(gs), int(F)),
                            self.device)
        arr = _lib.ptr_array(gs)
        timer = SpmmPlan.hop_timer
        with _lib.DeviceGuard(self.device):
            stream = _lib.stream_of(gx)
            t0 = timer.begin(torch.cuda.current_stream(self.device)) if timer else None
            rc = self.lib.cign_multihop_bwd(self.handle, len(gs), arr, int(F), _lib.ptr(gx),
                                            _lib.ptr(ws), ws.numel(), stream)
            if timer:
                # hop p (p = max..1) adds g_{p-1} when present: addend hops = grads[0..max-2]
                n_add = sum(1 for g in gs[:-1] if g is not None)
                timer.end(torch.cuda.current_stream(self.device), t0, "bwd", len(gs), n_add, int(F))
        _lib.check(rc, "cign_multihop_bwd")
        return gx


class GatPlan:
    """Native plan over the fixed GAT graph triple ((rowptr, col), (row, colptr), perm)."""

    def __init__(self, rowptr, col, row, colptr, perm):
        _lib.require_cuda("GatPlan")
        self.lib = _lib.load_library()
        self.device = rowptr.device
        self.rowptr, self.col = _as_i32(rowptr), _as_i32(col)
        self.row, self.colptr, self.perm = _as_i32(row), _as_i32(colptr), _as_i32(perm)
        self.n = int(self.rowptr.numel() - 1)
        self.n_cols = int(self.colptr.numel() - 1)
        self.nnz = int(self.col.numel())
        if self.row.numel() != self.nnz or self.perm.numel() != self.nnz:
            raise ValueError("GAT graph: CSR/CSC/perm sizes do not match")
        handle = ctypes.c_void_p()
        with _lib.DeviceGuard(self.device):
            rc = self.lib.cign_gat_plan_create_rect(
                self.n, self.n_cols, self.nnz, _lib.ptr(self.rowptr), _lib.ptr(self.col),
                _lib.ptr(self.colptr), _lib.ptr(self.row), _lib.ptr(self.perm), ctypes.byref(handle))
        _lib.check(rc, "cign_gat_plan_create")
        self.handle = handle

    def __del__(self):
        h = getattr(self, "handle", None)
        if h is not None and h.value:
            try:
                self.lib.cign_gat_plan_destroy(h)
            except Exception:
                pass
            self.handle = None

    def info(self) -> Dict[str, int]:
        arr = (ctypes.c_int64 * 8)()
        _lib.check(self.lib.cign_gat_plan_get_info(self.handle, arr), "cign_gat_plan_get_info")
        keys = ("n", "nnz", "heavy_rows", "heavy_cols", "max_row_len", "max_col_len",
                "row_segments", "col_segments")
        return {k: int(v) for k, v in zip(keys, arr)}


_CACHE_MAX = 16
_GAT_PLANS: "OrderedDict[Tuple[int, ...], GatPlan]" = OrderedDict()
_SPMM_PLANS: "OrderedDict[Tuple[int, ...], SpmmPlan]" = OrderedDict()


def _cache_put(cache, key, plan):
    cache[key] = plan
    cache.move_to_end(key)
    while len(cache) > _CACHE_MAX:
        cache.popitem(last=False)


def gat_plan_for(rowptr, col, row, colptr, perm) -> GatPlan:
    """Plan cached by the graph tensors' identity (data pointers and sizes).

    The cached plan keeps the caller's tensors alive, so their addresses
    cannot be recycled for a different graph while the entry exists."""
    key = (rowptr.data_ptr(), col.data_ptr(), row.data_ptr(), colptr.data_ptr(), perm.data_ptr(),
           int(rowptr.numel()), int(col.numel()), int(rowptr.device.index or 0))
    plan = _GAT_PLANS.get(key)
    if plan is None:
        plan = GatPlan(rowptr, col, row, colptr, perm)
        plan._keepalive = (rowptr, col, row, colptr, perm)
        _cache_put(_GAT_PLANS, key, plan)
    return plan


def spmm_plan_for(csr: torch.Tensor, csr_t: Optional[torch.Tensor]) -> SpmmPlan:
    """Plan cached by the sparse CSR tensors' identity (FixedCSRSpMMFunction)."""
    key = (csr.crow_indices().data_ptr(), csr.col_indices().data_ptr(), csr.values().data_ptr(),
           0 if csr_t is None else csr_t.values().data_ptr(), int(csr._nnz()))
    plan = _SPMM_PLANS.get(key)
    if plan is None:
        if csr_t is None:
            plan = SpmmPlan(csr.crow_indices(), csr.col_indices(), csr.values())
        else:
            plan = SpmmPlan(csr.crow_indices(), csr.col_indices(), csr.values(),
                            csr_t.crow_indices(), csr_t.col_indices(), csr_t.values())
        # Keep the sparse tensors alive with the plan so the cache key (their
        # storage addresses) cannot be reused by another tensor.
        plan._keepalive = (csr, csr_t)
        _cache_put(_SPMM_PLANS, key, plan)
    return plan
