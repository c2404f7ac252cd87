"""Graph-operator construction restated in numpy -- TEST INFRASTRUCTURE.

* ``normalized_adjacency``: generic_engine/train_cign.py:1558-1589
  (to_undirected -> add self loops -> degree over `col`, clamp(min=1),
  w = d^-1/2[row] * d^-1/2[col] in fp32 -> coalesce, duplicates summed).
* ``csr_of`` / ``csr_transpose``: prepare_fixed_csr_operator, model.py:149-186
  (coalesce = sort by (row, col) and sum duplicates; P^T by flipping the
  indices and coalescing again).
* ``gat_graph``: prepare_gat_edge_index (generic_engine/train_cign.py:1759-1771) followed by
  the destination-major CSR/CSC/perm layout read by the reference's GAT
  kernels (collapsed_gat_cuda.cu:227-248; generic_engine/model_cign.py:1117-1146).

The fp32 products are evaluated in float32 exactly as torch does, so the
values are bit-identical to the reference's, not merely close.
"""
from __future__ import annotations

import numpy as np


def to_undirected(edge_index: np.ndarray, n: int) -> np.ndarray:
    """Both directions of every edge, deduplicated and sorted by (row, col): the
    to_undirected step of build_sparse_normalized_adjacency
    (generic_engine/train_cign.py:1558-1589)."""
    row = np.asarray(edge_index[0], dtype=np.int64)
    col = np.asarray(edge_index[1], dtype=np.int64)
    key = np.unique(np.concatenate([row * n + col, col * n + row]))
    return np.stack([key // n, key % n])


def coalesce(row, col, val, n_rows: int, n_cols: int):
    """Sort by (row, col) and sum duplicate entries: torch COO coalesce, as
    prepare_fixed_csr_operator applies it (model.py:161-163, 176-183)."""
    key = np.asarray(row, np.int64) * n_cols + np.asarray(col, np.int64)
    order = np.argsort(key, kind="stable")
    key = key[order]
    val = np.asarray(val)[order]
    uniq, start = np.unique(key, return_index=True)
    summed = np.add.reduceat(val, start) if val.size else val
    return uniq // n_cols, uniq % n_cols, summed.astype(val.dtype, copy=False)


def normalized_adjacency(edge_index: np.ndarray, n: int, use_undirected: bool = True,
                         add_self_loop: bool = True):
    """Coalesced COO (row, col, val fp32) of D^-1/2 (A + I) D^-1/2
    (generic_engine/train_cign.py:1558-1589)."""
    ei = to_undirected(edge_index, n) if use_undirected else np.asarray(edge_index, np.int64)
    if add_self_loop:
        loops = np.arange(n, dtype=np.int64)
        ei = np.concatenate([ei, np.stack([loops, loops])], axis=1)
    row, col = ei[0], ei[1]
    deg = np.bincount(col, minlength=n).astype(np.float32)
    # torch evaluates pow(x, -0.5) on float32 CPU tensors as 1 / sqrt(x)
    dinv = (np.float32(1.0) / np.sqrt(np.maximum(deg, np.float32(1.0)))).astype(np.float32)
    w = (dinv[row] * dinv[col]).astype(np.float32)
    return coalesce(row, col, w, n, n)


def csr_of(row, col, val, n_rows: int):
    """CSR arrays (crow int64 [n_rows+1], col int64, val) of a coalesced COO:
    the to_sparse_csr conversion of prepare_fixed_csr_operator (model.py:149-186)."""
    crow = np.zeros(n_rows + 1, dtype=np.int64)
    np.cumsum(np.bincount(np.asarray(row, np.int64), minlength=n_rows), out=crow[1:])
    return crow, np.asarray(col, np.int64), np.asarray(val)


def csr_transpose(row, col, val, n: int):
    """CSR of P^T: flip the indices and coalesce (model.py:176-186)."""
    r, c, v = coalesce(col, row, val, n, n)
    return csr_of(r, c, v, n)


def prepare_gat_edge_index(edge_index: np.ndarray, n: int) -> np.ndarray:
    """Remove self-loops, then add exactly one per node
    (generic_engine/train_cign.py:1759-1771)."""
    ei = np.asarray(edge_index, np.int64)
    ei = ei[:, ei[0] != ei[1]]
    loops = np.arange(n, dtype=np.int64)
    return np.concatenate([ei, np.stack([loops, loops])], axis=1)


def gat_graph(edge_index_src_dst: np.ndarray, n: int):
    """((rowptr, col), (row, colptr), perm) for a PyG-style source->target edge
    list: rows are destinations (edge_index.flip(0), generic_engine/model_cign.py:1118),
    CSR sorted by (row, col) keeping duplicates, CSC a stable re-sort by
    column, perm[csc position] = CSR edge id."""
    dst = np.asarray(edge_index_src_dst[1], np.int64)
    src = np.asarray(edge_index_src_dst[0], np.int64)
    order = np.argsort(dst * n + src, kind="stable")
    r, c = dst[order], src[order]
    rowptr = np.zeros(n + 1, np.int64)
    np.cumsum(np.bincount(r, minlength=n), out=rowptr[1:])
    corder = np.argsort(c, kind="stable")
    colptr = np.zeros(n + 1, np.int64)
    np.cumsum(np.bincount(c, minlength=n), out=colptr[1:])
    return (rowptr, c), (r[corder], colptr), corder.astype(np.int64)
