"""Aggregate-first GAT layer (cign_gat_agg_fwd/_bwd + GEMMs) on the GPU vs the
CPU oracle of the reference order: in_feat = lin(x).view(N,H,C), then the
collapsed GAT (collapsed_gat_cuda.cu:52-545 restated in oracle.ops).  Forward,
edge statistics and the gradients of x, alpha_dst, alpha_src, lin.weight and
bias, with and without attention dropout, on graphs with hub rows/columns."""
import pytest
import torch

from cign_b200 import synth
from cign_b200.collapsed_gat import aggregate_first_with_plan, gat_agg_forward_raw
from cign_b200.graph_operator import prepare_gat_edge_index, to_graph_format
from cign_b200.plans import gat_plan_for
from oracle import ops
from tests.helpers import assert_parity

pytestmark = pytest.mark.gpu


def _plan(edge, n, dev):
    (rp, c), (r, cp), perm = to_graph_format(edge.flip(0), n)
    plan = gat_plan_for(rp.to(dev), c.to(dev), r.to(dev), cp.to(dev), perm.to(dev))
    return plan, rp, c


def _case(dev, edge, n, H, D, C, p, seed, slope=0.2):
    g = torch.Generator().manual_seed(31 * H + D + 7 * C)
    x = torch.randn(n, D, generator=g)
    W = torch.randn(H * C, D, generator=g) / D ** 0.5
    a_dst = torch.randn(n, H, generator=g)
    a_src = torch.randn(n, H, generator=g)
    bias = torch.randn(C, generator=g) * 0.1
    gy = torch.randn(n, C, generator=g)
    plan, rp, c = _plan(edge, n, dev)
    # oracle: lin first, then the collapsed GAT (CPU autograd)
    leaves = [t.clone().requires_grad_(True) for t in (x, a_dst, a_src, W, bias)]
    in_feat = (leaves[0] @ leaves[3].t()).view(n, H, C)
    out_o, pre_o, m_o, s_o = ops.gat_collapsed(leaves[1], leaves[2], rp, c, in_feat, leaves[4],
                                                slope, p, seed)
    grads_o = torch.autograd.grad(out_o, leaves, gy)
    # native, aggregate first
    ins = [t.to(dev).requires_grad_(True) for t in (x, a_dst, a_src, W, bias)]
    out = aggregate_first_with_plan(ins[0], ins[1], ins[2], ins[3], ins[4], plan, H, slope, p,
                                     seed)
    grads = torch.autograd.grad(out, ins, gy.to(dev))
    tag = f"n={n} H={H} D={D} C={C} p={p}"
    assert_parity(out, out_o.detach(), what=f"out {tag}")
    z, emax, esum = gat_agg_forward_raw(plan, ins[1].detach(), ins[2].detach(), ins[0].detach(),
                                        H, slope, p, seed)
    assert_parity(emax, m_o, what=f"edge_max {tag}")
    assert_parity(esum, s_o, what=f"edge_sum {tag}")
    for name, a, e in zip(("grad_x", "grad_attn_row", "grad_attn_col", "grad_weight", "grad_bias"),
                          grads, grads_o):
        assert_parity(a, e, what=f"{name} {tag}")
    return plan


def _random_graph(n, e, seed):
    g = torch.Generator().manual_seed(seed)
    src = torch.randint(0, n, (e,), generator=g)
    dst = torch.randint(0, n, (e,), generator=g)
    return prepare_gat_edge_index(torch.stack([src, dst]), n)


@pytest.mark.parametrize("H,D,C", [(1, 16, 16), (4, 64, 64), (4, 512, 512), (6, 132, 24),
                                   (8, 64, 128), (2, 300, 260)])
@pytest.mark.parametrize("p", [0.0, 0.5])
def test_agg_gat_vs_oracle(cuda, H, D, C, p):
    n = 300
    edge = _random_graph(n, 2400, seed=H * 11 + D)
    _case(cuda, edge, n, H, D, C, p, seed=987654321)


def test_agg_gat_hub_rows_and_columns(cuda):
    n = 1500
    edge = prepare_gat_edge_index(synth.powerlaw_graph(n, 12000, seed=9), n)
    plan = _case(cuda, edge, n, 4, 128, 64, 0.3, seed=77)
    info = plan.info()
    assert info["heavy_rows"] > 0 and info["heavy_cols"] > 0


def test_agg_gat_empty_rows(cuda):
    n = 64
    edge = torch.tensor([[0, 1, 2, 5, 5], [1, 2, 0, 5, 63]])  # most rows have no edges
    _case(cuda, edge, n, 2, 16, 8, 0.0, seed=1)


def test_agg_gat_deterministic(cuda):
    n = 1500
    edge = prepare_gat_edge_index(synth.powerlaw_graph(n, 12000, seed=3), n)
    plan, _, _ = _plan(edge, n, cuda)
    g = torch.Generator(device=cuda).manual_seed(0)
    x = torch.randn(n, 256, device=cuda, generator=g)
    a = torch.randn(n, 4, device=cuda, generator=g)
    z1, _, _ = gat_agg_forward_raw(plan, a, a, x, 4, 0.2, 0.4, 5)
    z2, _, _ = gat_agg_forward_raw(plan, a, a, x, 4, 0.2, 0.4, 5)
    assert torch.equal(z1, z2)


def test_agg_gat_kept_edge_weights_equal_recomputed(cuda):
    """The forward's edge weights handed to the backward (cign_gat_agg_fwd_w /
    _bwd_w) give the backward of the recomputing entry points bit for bit,
    with attention dropout and hub rows and columns."""
    from cign_b200.collapsed_gat import gat_agg_backward_raw, gat_agg_forward_keep_raw
    n, H, D = 1500, 4, 128
    edge = prepare_gat_edge_index(synth.powerlaw_graph(n, 12000, seed=21), n)
    plan, _, _ = _plan(edge, n, cuda)
    g = torch.Generator(device=cuda).manual_seed(5)
    x = torch.randn(n, D, device=cuda, generator=g)
    a_row = torch.randn(n, H, device=cuda, generator=g)
    a_col = torch.randn(n, H, device=cuda, generator=g)
    z1, m1, s1 = gat_agg_forward_raw(plan, a_row, a_col, x, H, 0.2, 0.4, 11)
    z2, m2, s2, wts = gat_agg_forward_keep_raw(plan, a_row, a_col, x, H, 0.2, 0.4, 11)
    assert torch.equal(z1, z2) and torch.equal(m1, m2) and torch.equal(s1, s2)
    gz = torch.randn(n, H * D, device=cuda, generator=g)
    gp = torch.randn(n, D, device=cuda, generator=g)
    ref = gat_agg_backward_raw(plan, a_row, a_col, x, m1, s1, gz, gp, 0.2, 0.4, 11)
    got = gat_agg_backward_raw(plan, a_row, a_col, x, m1, s1, gz, gp, 0.2, 0.4, 11, wts=wts)
    for r, o in zip(ref, got):
        assert torch.equal(r, o)
