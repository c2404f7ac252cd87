"""SpMM / k-hop propagation on the GPU vs the reference's outputs (golden)
and the CPU oracle.  Bit-exact index handling; fp32 within 1e-5 rel-L2."""
import numpy as np
import pytest
import torch

from cign_b200 import synth
from cign_b200.graph_operator import (FixedCSRSpMMFunction, build_sparse_normalized_adjacency,
                                      prepare_fixed_csr_operator, selected_sparse_powers)
from cign_b200.multihop_csr_pipeline import (GenericMultiHopCSRGraphOperator,
                                             HybridNative3TailCSRGraphOperator,
                                             MultiHopCSR3GraphOperator, prepare_multihop_csr_operator)
from cign_b200.plans import SpmmPlan
from oracle import graph as og
from oracle import ops
from tests.helpers import assert_parity, rel_l2

pytestmark = pytest.mark.gpu


def _coo(z, dev):
    n = int(z["n"])
    idx = torch.stack([torch.from_numpy(z["coo_row"]), torch.from_numpy(z["coo_col"])])
    return torch.sparse_coo_tensor(idx, torch.from_numpy(z["coo_val"]), (n, n)).to(dev)


def test_fixed_csr_golden(cuda, golden):
    z = golden("fixedcsr_random.npz")
    op = prepare_fixed_csr_operator(_coo(z, cuda))
    np.testing.assert_array_equal(op.csr.crow_indices().cpu().numpy(), z["crow"])
    np.testing.assert_array_equal(op.csr.col_indices().cpu().numpy(), z["col"])
    np.testing.assert_array_equal(op.csr_t.col_indices().cpu().numpy(), z["col_t"])
    x = torch.from_numpy(z["x"]).to(cuda).requires_grad_(True)
    y = FixedCSRSpMMFunction.apply(x, op.csr, op.csr_t)
    (y * torch.from_numpy(z["gy"]).to(cuda)).sum().backward()
    assert_parity(y.detach(), z["y"], what="spmm fwd")
    assert_parity(x.grad, z["gx"], what="spmm bwd (P^T)")


@pytest.mark.parametrize("name,powers,cls", [
    ("p123", (1, 2, 3), MultiHopCSR3GraphOperator),
    ("p1248", (1, 2, 4, 8), HybridNative3TailCSRGraphOperator),
    ("p0_2_5", (0, 2, 5), HybridNative3TailCSRGraphOperator),
])
def test_multihop_golden(cuda, golden, name, powers, cls):
    z = golden("multihop_circulant.npz")
    base = prepare_fixed_csr_operator(_coo(z, cuda))
    d = int(z[f"{name}_x"].shape[1])
    op = prepare_multihop_csr_operator(base, dense_cols=d, powers=powers)
    assert isinstance(op, cls)
    x = torch.from_numpy(z[f"{name}_x"]).to(cuda).requires_grad_(True)
    out = selected_sparse_powers(op, x, powers)
    loss = 0
    for p in powers:
        if p == 0:
            assert out[0] is x
            continue
        assert_parity(out[p].detach(), z[f"{name}_y{p}"], what=f"P^{p}")
        loss = loss + (out[p] * torch.from_numpy(z[f"{name}_g{p}"]).to(cuda)).sum()
    loss.backward()
    assert_parity(x.grad, z[f"{name}_gx"], what="grad x")


def _powerlaw_operator(n, e, seed, dev):
    edge = synth.powerlaw_graph(n, e, seed=seed)
    _, adj = build_sparse_normalized_adjacency(edge, n)
    r, c, v = og.normalized_adjacency(edge.numpy(), n)
    P = ops.csr_tensor(*og.csr_of(r, c, v, n), n, n)
    return prepare_fixed_csr_operator(adj.to(dev)), P


@pytest.mark.parametrize("F", [1, 3, 12, 64, 128, 200, 512, 1024, 1100])
def test_spmm_shapes_vs_oracle(cuda, F):
    """Every dispatch configuration (scalar/float4, 8/16/32 lanes, 1-8 vectors
    per lane, >1024 feature tiles) on a power-law graph with hub rows."""
    n = 4000
    base, P = _powerlaw_operator(n, 30000, 11, cuda)
    plan = SpmmPlan(base.csr.crow_indices(), base.csr.col_indices(), base.csr.values())
    assert plan.info()["heavy_rows"] > 0  # the hub-row segment path is exercised
    g = torch.Generator().manual_seed(F)
    x = torch.randn(n, F, generator=g)
    y = plan.spmm(x.to(cuda))
    assert_parity(y, torch.sparse.mm(P, x), what=f"F={F}")
    add = torch.randn(n, F, generator=g)
    y2 = plan.spmm(x.to(cuda), transpose=True, addend=add.to(cuda))
    assert_parity(y2, torch.sparse.mm(P, x) + add, what=f"F={F} transposed + addend")


def test_spmm_unaligned_and_nonsymmetric(cuda):
    torch.manual_seed(0)
    n, e = 700, 9000
    row = torch.randint(0, n, (e,))
    col = torch.randint(0, n, (e,))
    val = torch.rand(e)
    coo = torch.sparse_coo_tensor(torch.stack([row, col]), val, (n, n)).coalesce()
    base = prepare_fixed_csr_operator(coo.to(cuda))
    Pc = coo.to_sparse_csr()
    PTc = coo.t().coalesce().to_sparse_csr()
    buf = torch.randn(n * 64 + 1)
    xg = buf.to(cuda)[1:1 + n * 64].view(n, 64)  # 4-byte offset: scalar path
    assert xg.data_ptr() % 16 != 0
    y = FixedCSRSpMMFunction.apply(xg, base.csr, base.csr_t)
    assert_parity(y, torch.sparse.mm(Pc, buf[1:1 + n * 64].view(n, 64)), what="unaligned")
    xg2 = torch.randn(n, 32)
    plan = SpmmPlan(base.csr.crow_indices(), base.csr.col_indices(), base.csr.values(),
                    base.csr_t.crow_indices(), base.csr_t.col_indices(), base.csr_t.values())
    assert not plan.symmetric
    assert_parity(plan.spmm(xg2.to(cuda), transpose=True), torch.sparse.mm(PTc, xg2), what="P^T")


def test_spmm_empty_rows_and_empty_graph(cuda):
    n = 50
    row = torch.tensor([0, 0, 3, 49])
    col = torch.tensor([1, 2, 3, 0])
    val = torch.tensor([1.0, 2.0, 3.0, 4.0])
    coo = torch.sparse_coo_tensor(torch.stack([row, col]), val, (n, n)).coalesce()
    base = prepare_fixed_csr_operator(coo.to(cuda))
    x = torch.randn(n, 16)
    y = FixedCSRSpMMFunction.apply(x.to(cuda), base.csr, base.csr_t)
    assert_parity(y, torch.sparse.mm(coo, x), what="sparse rows")
    assert bool((y[4:49] == 0).all())
    empty = torch.sparse_coo_tensor(torch.zeros(2, 0, dtype=torch.long), torch.zeros(0), (8, 8))
    base0 = prepare_fixed_csr_operator(empty.to(cuda))
    y0 = FixedCSRSpMMFunction.apply(torch.randn(8, 4, device=cuda), base0.csr, base0.csr_t)
    assert bool((y0 == 0).all())


def test_multihop_deterministic_and_generic_k(cuda):
    n = 3000
    base, P = _powerlaw_operator(n, 25000, 5, cuda)
    for powers in [(1,), (1, 2), (2, 5, 8), (1, 2, 3, 4, 5, 6, 7, 8)]:
        op = GenericMultiHopCSRGraphOperator(base, dense_cols=96, powers=powers)
        x = torch.randn(n, 96)
        xg = x.to(cuda).requires_grad_(True)
        out = selected_sparse_powers(op, xg, powers)
        gs = {p: torch.randn(n, 96) for p in powers}
        loss = sum((out[p] * gs[p].to(cuda)).sum() for p in powers)
        loss.backward()
        xr = x.clone().requires_grad_(True)
        ref = ops.multihop(P, P, xr, powers)
        sum((ref[p] * gs[p]).sum() for p in powers).backward()
        for p in powers:
            assert_parity(out[p].detach(), ref[p].detach(), what=f"{powers} P^{p}")
        assert_parity(xg.grad, xr.grad, what=f"{powers} grad")
        # bitwise determinism
        out2 = selected_sparse_powers(op, xg.detach(), powers)
        for p in powers:
            assert torch.equal(out2[p], out[p].detach())


def test_cfg2_scale_properties(cuda):
    """Full cfg2 size (N=24,492, F=1024): adjoint identity <Px,y> = <x,P^T y>
    (P symmetric), linearity, and against the oracle on a row sample."""
    cfg = synth.CONFIGS["cfg2"]
    edge = synth.make_edges(cfg)
    n = cfg.num_nodes
    _, adj = build_sparse_normalized_adjacency(edge, n)
    base = prepare_fixed_csr_operator(adj.to(cuda))
    op = prepare_multihop_csr_operator(base, dense_cols=1024)
    plan = op.plan.spmm
    assert plan.symmetric and plan.info()["heavy_rows"] > 0
    g = torch.Generator(device=cuda).manual_seed(0)
    x = torch.randn(n, 1024, device=cuda, generator=g)
    yv = torch.randn(n, 1024, device=cuda, generator=g)
    px = plan.spmm(x)
    pty = plan.spmm(yv, transpose=True)
    lhs = (px.double() * yv.double()).sum()
    rhs = (x.double() * pty.double()).sum()
    assert abs(float(lhs - rhs)) <= 1e-5 * float((px.double().abs() * yv.double().abs()).sum())
    a, b = 0.75, -1.25
    lin = plan.spmm(a * x + b * yv)
    assert rel_l2(lin, a * px + b * plan.spmm(yv)) < 1e-5
    r, c, v = og.normalized_adjacency(edge.numpy(), n)
    P = ops.csr_tensor(*og.csr_of(r, c, v, n), n, n)
    sample = torch.arange(0, n, 97)
    ref = torch.sparse.mm(P, x.cpu())[sample]
    assert_parity(px.cpu()[sample], ref, what="cfg2 row sample")
    y1, y2, y3 = op.plan.forward3(x)
    assert_parity(y2.cpu()[sample], torch.sparse.mm(P, y1.cpu())[sample], what="hop 2")


@pytest.mark.parametrize("d", [256, 512])
def test_multihop_split_input_equals_concatenated(cuda, d):
    """cign_multihop_fwd_split (hop 1 reads [H | C] as two matrices) gives the
    hops of the concatenated input bit for bit, hub rows included."""
    n = 4000
    base, _ = _powerlaw_operator(n, 30000, 13, cuda)
    plan = SpmmPlan(base.csr.crow_indices(), base.csr.col_indices(), base.csr.values())
    assert plan.info()["heavy_rows"] > 0
    g = torch.Generator().manual_seed(d)
    h = torch.randn(n, d, generator=g).to(cuda)
    c = torch.randn(n, d, generator=g).to(cuda)
    ys = plan.forward_split(h, c, 3)
    ref = plan.forward(torch.cat([h, c], 1), 3)
    for p in range(3):
        assert torch.equal(ys[p], ref[p]), p
