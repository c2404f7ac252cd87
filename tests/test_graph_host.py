"""Host-side graph preparation of the product (torch ops) against the numpy
oracle restatement: bit-exact CSR / CSR^T / CSC / perm and fp32 operator
values.  CPU only."""
import numpy as np
import torch

from cign_b200 import synth
from cign_b200.graph_operator import (build_sparse_normalized_adjacency, prepare_fixed_csr_operator,
                                      prepare_gat_edge_index, to_graph_format)
from oracle import graph as og


def _check_graph(edge, n):
    ei_used, adj = build_sparse_normalized_adjacency(edge, n)
    op = prepare_fixed_csr_operator(adj)
    r, c, v = og.normalized_adjacency(edge.numpy(), n)
    crow, col, val = og.csr_of(r, c, v, n)
    np.testing.assert_array_equal(op.csr.crow_indices().numpy(), crow)
    np.testing.assert_array_equal(op.csr.col_indices().numpy(), col)
    np.testing.assert_array_equal(op.csr.values().numpy(), val)  # bit-exact fp32
    crow_t, col_t, val_t = og.csr_transpose(r, c, v, n)
    np.testing.assert_array_equal(op.csr_t.crow_indices().numpy(), crow_t)
    np.testing.assert_array_equal(op.csr_t.col_indices().numpy(), col_t)
    np.testing.assert_array_equal(op.csr_t.values().numpy(), val_t)
    gat_e = prepare_gat_edge_index(ei_used, n)
    (rp, cc), (rr, cp), perm = to_graph_format(gat_e.flip(0), n)
    (rp_o, cc_o), (rr_o, cp_o), perm_o = og.gat_graph(og.prepare_gat_edge_index(ei_used.numpy(), n), n)
    for a, b in ((rp, rp_o), (cc, cc_o), (rr, rr_o), (cp, cp_o), (perm, perm_o)):
        np.testing.assert_array_equal(a.numpy(), b)
    # perm consistency: CSC position -> CSR edge with the same (row, col)
    row_of_edge = np.repeat(np.arange(n), np.diff(rp.numpy()))
    np.testing.assert_array_equal(row_of_edge[perm.numpy()], rr.numpy())
    np.testing.assert_array_equal(cc.numpy()[perm.numpy()],
                                  np.repeat(np.arange(n), np.diff(cp.numpy())))
    return op


def test_er_graph_cfg1_shape():
    cfg = synth.CONFIGS["cfg1"]
    edge = synth.make_edges(cfg)
    assert edge.shape == (2, 8000)
    op = _check_graph(edge, cfg.num_nodes)
    # symmetric operator: CSR(P^T) is CSR(P) bit for bit
    assert torch.equal(op.csr.values(), op.csr_t.values())


def test_powerlaw_graph_small():
    edge = synth.powerlaw_graph(3000, 20000, seed=3)
    assert edge.shape == (2, 20000)
    assert bool((edge[0] != edge[1]).all())
    key = edge[0] * 3000 + edge[1]
    assert key.unique().numel() == 20000
    _check_graph(edge, 3000)


def test_rmat_graph_small():
    edge = synth.rmat_graph(5000, 30000, seed=1)
    assert edge.shape == (2, 30000)
    assert int(edge.max()) < 5000
    _check_graph(edge, 5000)


def test_isolated_nodes_and_duplicates():
    n = 10
    edge = torch.tensor([[0, 0, 1, 3, 3], [1, 1, 0, 3, 4]])  # duplicate, reverse, self loop
    _check_graph(edge, n)


def test_split_masks():
    tr, va, te = synth.random_ratio_split(101, 0.5, 0.25, 0.25, 42)
    assert int(tr.sum()) == 50 and int(va.sum()) == 25 and int(te.sum()) == 26
    assert not bool((tr & va).any() or (tr & te).any() or (va & te).any())
