"""Fixed graph operator P: CSR(P)/CSR(P^T) construction, single-SpMM autograd
and the hop dispatcher -- the pieces of the reference's model.py that sit on
the propagation path (model.py:57-252; duplicate in generic_engine/
model_cign.py:109-304), plus the operator builder of the training script
(generic_engine/train_cign.py:1558-1589).

Index construction follows the reference exactly (torch COO coalesce, then
``flip`` + coalesce for P^T), so CSR arrays are bit-identical to what the
reference builds; the SpMM itself runs on the native sm_100a kernel.
"""
from __future__ import annotations

import torch

from .multihop_csr_pipeline import (
    GenericMultiHopCSRGraphOperator,
    HybridNative3TailCSRGraphOperator,
    MultiHopCSR3GraphOperator,
    generic_multihop_csr,
    hybrid_native3_tail_csr,
    multihop_csr3,
)
from .plans import spmm_plan_for


class FixedCSRSpMMFunction(torch.autograd.Function):
    """Y = P X; grad_X = P^T grad_Y (model.py:57-106), on the native SpMM."""

    @staticmethod
    def forward(ctx, X: torch.Tensor, operator_csr: torch.Tensor, operator_t_csr: torch.Tensor):
        if operator_csr.layout != torch.sparse_csr:
            raise TypeError(f"operator_csr must be sparse CSR, got {operator_csr.layout}")
        if operator_t_csr.layout != torch.sparse_csr:
            raise TypeError(f"operator_t_csr must be sparse CSR, got {operator_t_csr.layout}")
        if operator_csr.dtype != operator_t_csr.dtype:
            raise TypeError(
                f"CSR(P) and CSR(P^T) must share dtype, got {operator_csr.dtype} and {operator_t_csr.dtype}"
            )
        if not X.is_cuda:
            raise RuntimeError("FixedCSRSpMMFunction requires CUDA tensors (no CPU fallback).")
        plan = spmm_plan_for(operator_csr, operator_t_csr)
        ctx.plan = plan
        ctx.input_dtype = X.dtype
        return plan.spmm(X.to(dtype=torch.float32).contiguous(), transpose=False)

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        grad_X = ctx.plan.spmm(grad_output.to(dtype=torch.float32).contiguous(), transpose=True)
        if grad_X.dtype != ctx.input_dtype:
            grad_X = grad_X.to(ctx.input_dtype)
        return grad_X, None, None


class FixedCSRGraphOperator:
    """Immutable cache holding CSR(P) and CSR(P^T) (model.py:109-146)."""

    __slots__ = ("csr", "csr_t", "shape", "nnz", "dtype", "device", "info")

    def __init__(self, csr: torch.Tensor, csr_t: torch.Tensor):
        self.csr = csr
        self.csr_t = csr_t
        self.shape = tuple(csr.shape)
        self.nnz = int(csr.values().numel())
        self.dtype = csr.dtype
        self.device = csr.device
        self.info = {
            "layout": "csr",
            "shape": self.shape,
            "nnz": self.nnz,
            "dtype": str(self.dtype),
            "device": str(self.device),
        }


def _clone_csr_storage(csr: torch.Tensor) -> torch.Tensor:
    return torch.sparse_csr_tensor(
        csr.crow_indices().clone().contiguous(),
        csr.col_indices().clone().contiguous(),
        csr.values().clone().contiguous(),
        size=csr.shape,
        dtype=csr.dtype,
        device=csr.device,
    )


@torch.no_grad()
def prepare_fixed_csr_operator(operator: torch.Tensor) -> FixedCSRGraphOperator:
    """COO/CSR operator -> cached CSR(P), CSR(P^T) (model.py:149-186)."""
    if not isinstance(operator, torch.Tensor):
        raise TypeError(f"operator must be a torch.Tensor, got {type(operator)!r}")
    if operator.dim() != 2 or operator.size(0) != operator.size(1):
        raise ValueError(f"Expected a square 2-D graph operator, got shape={tuple(operator.shape)}")
    if operator.layout == torch.sparse_coo:
        coo = operator.coalesce()
    elif operator.layout == torch.sparse_csr:
        coo = operator.to_sparse_coo().coalesce()
    else:
        raise TypeError(
            "FixedCSRSpMM expects a sparse COO or sparse CSR graph operator; "
            f"got layout={operator.layout}."
        )
    csr = _clone_csr_storage(coo.to_sparse_csr())
    idx_t = coo.indices().flip(0).contiguous()
    coo_t = torch.sparse_coo_tensor(idx_t, coo.values(), size=(coo.size(1), coo.size(0)),
                                    dtype=coo.dtype, device=coo.device).coalesce()
    csr_t = _clone_csr_storage(coo_t.to_sparse_csr())
    return FixedCSRGraphOperator(csr=csr, csr_t=csr_t)


def fixed_sparse_mm(operator, X: torch.Tensor) -> torch.Tensor:
    """One P @ X (model.py:202-213)."""
    if isinstance(operator, FixedCSRGraphOperator):
        return FixedCSRSpMMFunction.apply(X, operator.csr, operator.csr_t)
    raise TypeError(f"Unsupported graph operator type: {type(operator)!r}")


def selected_sparse_powers(operator, X: torch.Tensor, powers):
    """dict{power: P^power X} for the requested powers (model.py:216-252)."""
    requested = {int(power) for power in powers}
    if not requested:
        raise ValueError("powers cannot be empty.")
    if min(requested) < 0:
        raise ValueError(f"Graph-operator powers must be non-negative, got {sorted(requested)}.")
    outputs = {}
    if 0 in requested:
        outputs[0] = X
    if hasattr(operator, "powers") and callable(operator.powers):
        # a row-partitioned operator (cign_b200.distributed.DistMultiHop)
        return operator.powers(X, sorted(requested))
    if isinstance(operator, MultiHopCSR3GraphOperator) and requested == {1, 2, 3}:
        y1, y2, y3 = multihop_csr3(operator, X)
        outputs[1], outputs[2], outputs[3] = y1, y2, y3
        return outputs
    if isinstance(operator, HybridNative3TailCSRGraphOperator):
        outputs.update(hybrid_native3_tail_csr(operator, X))
        return outputs
    if isinstance(operator, GenericMultiHopCSRGraphOperator):
        outputs.update(generic_multihop_csr(operator, X))
        return outputs
    current = X
    for power in range(1, max(requested) + 1):
        current = fixed_sparse_mm(operator, current)
        if power in requested:
            outputs[power] = current
    return outputs


@torch.no_grad()
def to_undirected(edge_index: torch.Tensor, num_nodes: int) -> torch.Tensor:
    """Symmetrise and coalesce an edge list: the union of (u,v) and (v,u),
    sorted by (row, col) with duplicates removed (the semantics of
    torch_geometric.utils.to_undirected that build_sparse_normalized_adjacency
    relies on, generic_engine/train_cign.py:1571-1572)."""
    row, col = edge_index[0], edge_index[1]
    r = torch.cat([row, col])
    c = torch.cat([col, row])
    key = torch.unique(r * int(num_nodes) + c)
    return torch.stack([key // int(num_nodes), key % int(num_nodes)], dim=0)


@torch.no_grad()
def build_sparse_normalized_adjacency(edge_index: torch.Tensor, num_nodes: int,
                                      use_undirected: bool = True, add_self_loop: bool = True):
    """A_norm = D^{-1/2} (A + I) D^{-1/2} as a coalesced fp32 COO tensor
    (generic_engine/train_cign.py:1558-1589): degree counted over `col`,
    clamped at 1, weights deg^-1/2[row] * deg^-1/2[col], duplicates summed by
    coalesce.  Returns (edge_index_used, adjacency)."""
    if use_undirected:
        edge_index = to_undirected(edge_index, num_nodes)
    if add_self_loop:
        loops = torch.arange(num_nodes, device=edge_index.device, dtype=edge_index.dtype)
        edge_index = torch.cat([edge_index, torch.stack([loops, loops])], dim=1)
    row, col = edge_index
    deg = torch.zeros(num_nodes, dtype=torch.float32, device=edge_index.device)
    deg.scatter_add_(0, col, torch.ones_like(col, dtype=torch.float32))
    deg_inv_sqrt = deg.clamp(min=1.0).pow(-0.5)
    edge_weight = deg_inv_sqrt[row] * deg_inv_sqrt[col]
    adjacency = torch.sparse_coo_tensor(indices=edge_index, values=edge_weight,
                                        size=(num_nodes, num_nodes), dtype=torch.float).coalesce()
    return edge_index, adjacency


@torch.no_grad()
def prepare_gat_edge_index(edge_index: torch.Tensor, num_nodes: int) -> torch.Tensor:
    """Remove self-loops, then add exactly one per node (generic_engine/train_cign.py:1759-1771)."""
    mask = edge_index[0] != edge_index[1]
    ei = edge_index[:, mask]
    loops = torch.arange(num_nodes, device=edge_index.device, dtype=edge_index.dtype)
    return torch.cat([ei, torch.stack([loops, loops])], dim=1)


@torch.no_grad()
def to_graph_format(edge_index_dst_src: torch.Tensor, num_nodes: int):
    """CSR/CSC/perm of a destination-major edge list (row 0 = destination):

    * CSR: edges sorted by (row, col) with duplicates kept, rowptr int32;
    * CSC: the CSR edges stably re-sorted by column, colptr int32;
    * perm[csc position] = CSR edge id.

    This is the convention the reference's GAT kernels read
    (collapsed_gat_cuda.cu:227-248, generic_engine/model_cign.py:1117-1146); the PyG helper it
    obtains it from is not vendored, so the order is defined here.
    Returns ((rowptr, col), (row, colptr), perm), all int32 and contiguous.
    """
    n = int(num_nodes)
    r = edge_index_dst_src[0].to(torch.int64)
    c = edge_index_dst_src[1].to(torch.int64)
    key = r * n + c
    order = torch.sort(key, stable=True).indices
    r, c = r[order], c[order]
    rowptr = torch.zeros(n + 1, dtype=torch.int64, device=r.device)
    rowptr[1:] = torch.cumsum(torch.bincount(r, minlength=n), 0)
    corder = torch.sort(c, stable=True).indices
    row_csc = r[corder]
    colptr = torch.zeros(n + 1, dtype=torch.int64, device=r.device)
    colptr[1:] = torch.cumsum(torch.bincount(c, minlength=n), 0)
    as32 = lambda t: t.to(torch.int32).clone().contiguous()  # noqa: E731
    return (as32(rowptr), as32(c)), (as32(row_csc), as32(colptr)), as32(corder)
