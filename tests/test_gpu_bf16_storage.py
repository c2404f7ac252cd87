"""bf16 feature storage with fp32 accumulation (the large-graph configuration
stores node features as bf16; the reference's sparse path is fp32 only, so
the oracle is the fp32 computation on the widened inputs).

bf16 -> fp32 products equal the fp32 kernels on the widened features bit for
bit (same edge order, same fp32 FMAs); bf16 outputs equal the fp32 result
rounded to nearest even; and the fp32 results are within 1e-5 (rel-L2) of
the CPU oracle on the widened inputs."""
import pytest
import torch

from cign_b200 import collapsed_gat, synth
from cign_b200.graph_operator import (build_sparse_normalized_adjacency,
                                      prepare_fixed_csr_operator, prepare_gat_edge_index,
                                      to_graph_format)
from cign_b200.multihop_csr_pipeline import _csr_parts_int32
from cign_b200.plans import SpmmPlan, gat_plan_for
from oracle import ops
from tests.helpers import assert_parity

pytestmark = pytest.mark.gpu


def _operator(dev, n=3000, e=30000, seed=5):
    edge = synth.powerlaw_graph(n, e, seed=seed).to(dev)
    ei, adj = build_sparse_normalized_adjacency(edge, n)
    base = prepare_fixed_csr_operator(adj)
    return ei, base, SpmmPlan(*_csr_parts_int32(base.csr))


@pytest.mark.parametrize("F", [1024, 512, 136, 8])
def test_spmm_bf16_equals_fp32_on_widened_input(cuda, F):
    _, base, plan = _operator(cuda)
    assert plan.info()["heavy_rows"] > 0  # hub rows take the segment + combine path
    g = torch.Generator(device=cuda).manual_seed(F)
    xb = torch.randn(base.csr.size(0), F, device=cuda, generator=g).to(torch.bfloat16)
    ref = plan.spmm(xb.float())
    y32 = plan.spmm_bf16(xb, out_dtype=torch.float32)
    assert torch.equal(y32, ref)
    y16 = plan.spmm_bf16(xb, out_dtype=torch.bfloat16)
    assert torch.equal(y16, ref.to(torch.bfloat16))
    P = ops.csr_tensor(base.csr.crow_indices().cpu(), base.csr.col_indices().cpu(),
                       base.csr.values().cpu(), base.csr.size(0), base.csr.size(1))
    assert_parity(y32, torch.sparse.mm(P, xb.float().cpu()), what=f"spmm_bf16 F={F}")


def test_spmm_bf16_transpose_rectangular(cuda):
    """A rectangular, non-symmetric operator and its transpose."""
    g = torch.Generator().manual_seed(1)
    rows, cols, nnz = 700, 1100, 9000
    r = torch.randint(0, rows, (nnz,), generator=g)
    c = torch.randint(0, cols, (nnz,), generator=g)
    A = torch.sparse_coo_tensor(torch.stack([r, c]), torch.rand(nnz, generator=g),
                                (rows, cols)).coalesce()
    At = A.t().coalesce()
    a, at = A.to_sparse_csr(), At.to_sparse_csr()
    plan = SpmmPlan(*(t.to(cuda) for t in (a.crow_indices(), a.col_indices(), a.values(),
                                           at.crow_indices(), at.col_indices(), at.values())),
                    cols=cols)
    xb = torch.randn(cols, 64, generator=g).to(torch.bfloat16).to(cuda)
    assert torch.equal(plan.spmm_bf16(xb, torch.float32), plan.spmm(xb.float()))
    gb = torch.randn(rows, 64, generator=g).to(torch.bfloat16).to(cuda)
    assert torch.equal(plan.spmm_bf16(gb, torch.float32, transpose=True),
                       plan.spmm(gb.float(), transpose=True))


def test_multihop_bf16_chain(cuda):
    """Every hop stored as bf16: hop p = bf16(P . widen(hop p-1))."""
    _, base, plan = _operator(cuda, n=2000, e=16000, seed=8)
    g = torch.Generator(device=cuda).manual_seed(2)
    xb = torch.randn(2000, 256, device=cuda, generator=g).to(torch.bfloat16)
    ys = plan.forward_bf16(xb, 3)
    prev = xb
    for p, y in enumerate(ys, 1):
        want = plan.spmm(prev.float()).to(torch.bfloat16)
        assert y.dtype == torch.bfloat16 and torch.equal(y, want), f"hop {p}"
        prev = want


@pytest.mark.parametrize("H,D,p", [(4, 512, 0.5), (6, 64, 0.0), (8, 128, 0.3)])
def test_gat_aggregate_bf16_equals_fp32_on_widened_input(cuda, H, D, p):
    n = 1500
    edge = synth.powerlaw_graph(n, 12000, seed=H + D)
    ei = prepare_gat_edge_index(edge, n)
    (rp, c), (r, cp), perm = to_graph_format(ei.flip(0), n)
    plan = gat_plan_for(*(t.to(cuda) for t in (rp, c, r, cp, perm)))
    g = torch.Generator(device=cuda).manual_seed(H * D)
    xb = torch.randn(n, D, device=cuda, generator=g).to(torch.bfloat16)
    a_row = torch.randn(n, H, device=cuda, generator=g)
    a_col = torch.randn(n, H, device=cuda, generator=g)
    z16, m16, s16 = collapsed_gat.gat_agg_forward_raw(plan, a_row, a_col, xb, H, 0.2, p, 99)
    z32, m32, s32 = collapsed_gat.gat_agg_forward_raw(plan, a_row, a_col, xb.float(), H, 0.2, p,
                                                      99)
    assert torch.equal(z16, z32) and torch.equal(m16, m32) and torch.equal(s16, s32)
