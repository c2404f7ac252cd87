"""Collapsed GAT, attention logits and head-mean side op on the GPU vs the
CPU oracle: forward, all gradients, dropout masks bit for bit."""
import numpy as np
import pytest
import torch

from cign_b200 import collapsed_gat, synth
from cign_b200.collapsed_gat import collapsed_gat_mean_bias_silu, gat_dropout_mask
from cign_b200.fused_gat_sideops import fused_attention_logits, fused_head_mean_bias_silu
from cign_b200.graph_operator import prepare_gat_edge_index, to_graph_format
from cign_b200.plans import gat_plan_for
from oracle import ops, rng
from tests.helpers import assert_parity

pytestmark = pytest.mark.gpu


def _graph(edge, n, dev):
    (rp, c), (r, cp), perm = to_graph_format(edge.flip(0), n)
    return ((rp.to(dev), c.to(dev)), (r.to(dev), cp.to(dev)), perm.to(dev)), (rp, c)


def _gat_case(dev, n, H, C, edge, p, seed=0, slope=0.2):
    g = torch.Generator().manual_seed(1000 * H + C)
    x = torch.randn(n, H, C, generator=g)
    a_row = torch.randn(n, H, generator=g)
    a_col = torch.randn(n, H, generator=g)
    bias = torch.randn(C, generator=g) * 0.1
    gy = torch.randn(n, C, generator=g)
    gpu_graph, (rp, c) = _graph(edge, n, dev)
    # oracle (CPU autograd)
    leaves = [t.clone().requires_grad_(True) for t in (a_row, a_col, x, bias)]
    out_o, pre_o, m_o, s_o = ops.gat_collapsed(leaves[0], leaves[1], rp, c, leaves[2], leaves[3],
                                                slope, p, seed)
    grads_o = torch.autograd.grad(out_o, leaves, gy)
    # native
    plan = gat_plan_for(gpu_graph[0][0], gpu_graph[0][1], gpu_graph[1][0], gpu_graph[1][1],
                        gpu_graph[2])
    out, pre, emax, esum = collapsed_gat.gat_forward_raw(
        plan, a_row.to(dev), a_col.to(dev), x.to(dev), bias.to(dev), slope, p, seed)
    gfeat, grow, gcol, gbias = collapsed_gat.gat_backward_raw(
        plan, a_row.to(dev), a_col.to(dev), x.to(dev), pre, emax, esum, gy.to(dev), slope, p, seed)
    tag = f"n={n} H={H} C={C} p={p}"
    assert_parity(out, out_o.detach(), what=f"out {tag}")
    assert_parity(pre, pre_o.detach(), what=f"pre {tag}")
    assert_parity(emax, m_o, what=f"edge_max {tag}")
    assert_parity(esum, s_o, what=f"edge_sum {tag}")
    for name, a, e in (("grad_attn_row", grow, grads_o[0]), ("grad_attn_col", gcol, grads_o[1]),
                       ("grad_feat", gfeat, grads_o[2]), ("grad_bias", gbias, grads_o[3])):
        assert_parity(a, e, what=f"{name} {tag}")
    return plan


def _random_graph(n, e, seed):
    g = torch.Generator().manual_seed(seed)
    src = torch.randint(0, n, (e,), generator=g)
    dst = torch.randint(0, n, (e,), generator=g)
    return prepare_gat_edge_index(torch.stack([src, dst]), n)


@pytest.mark.parametrize("H,C", [(1, 16), (4, 16), (6, 24), (2, 6), (4, 300), (4, 512), (8, 64),
                                 (3, 1100)])
@pytest.mark.parametrize("p", [0.0, 0.5])
def test_gat_vs_oracle(cuda, H, C, p):
    n = 300
    edge = _random_graph(n, 2400, seed=H * 7 + C)
    _gat_case(cuda, n, H, C, edge, p, seed=123456789)


def test_gat_hub_rows_and_columns(cuda):
    """Rows and columns with > 128 edges take the one-CTA-per-row path."""
    n = 1500
    edge = prepare_gat_edge_index(synth.powerlaw_graph(n, 12000, seed=9), n)
    plan = _gat_case(cuda, n, 4, 64, edge, 0.3, seed=77)
    info = plan.info()
    assert info["heavy_rows"] > 0 and info["heavy_cols"] > 0


def test_gat_empty_rows(cuda):
    n = 40
    edge = torch.tensor([[1, 2, 3, 5, 5], [0, 0, 1, 7, 7]])  # duplicates kept, most rows empty
    _gat_case(cuda, n, 2, 8, edge, 0.0)


def test_gat_dropout_mask_bit_exact(cuda):
    for seed, p in ((0x1234_5678_9ABC, 0.32), (rng.gat_seed(42, 3), 0.5), (7, 0.05)):
        m = gat_dropout_mask(5000, 6, p, seed, cuda).cpu().numpy().reshape(-1)
        np.testing.assert_array_equal(m.astype(bool), rng.gat_keep_mask(seed, 30000, p))


def test_gat_module_api_seed_stream(cuda):
    """collapsed_gat_mean_bias_silu draws seeds like the reference
    (collapsed_gat.py:201-211): counter advances only when attn_drop > 0."""
    n, H, C = 200, 4, 32
    edge = _random_graph(n, 1500, seed=4)
    gpu_graph, (rp, c) = _graph(edge, n, cuda)
    torch.manual_seed(42)
    x = torch.randn(n, H, C, device=cuda)
    a_row = torch.randn(n, H, device=cuda)
    a_col = torch.randn(n, H, device=cuda)
    bias = torch.zeros(C, device=cuda)
    start = next(collapsed_gat._CALL_COUNTER) + 1  # counter state after this probe
    csr, csc, perm = gpu_graph
    collapsed_gat_mean_bias_silu(a_row, a_col, csr, csc, perm, 0.2, x, bias, 0.0)  # no advance
    y = collapsed_gat_mean_bias_silu(a_row, a_col, csr, csc, perm, 0.2, x, bias, 0.4)
    seed = rng.gat_seed(torch.initial_seed(), start)
    ref, _, _, _ = ops.gat_collapsed(a_row.cpu(), a_col.cpu(), rp, c, x.cpu(), bias.cpu(), 0.2, 0.4,
                                     seed)
    assert_parity(y, ref, what="seeded call")


@pytest.mark.parametrize("H,C", [(4, 512), (6, 256), (3, 10)])
def test_attention_logits_and_head_silu(cuda, H, C):
    n = 257
    g = torch.Generator().manual_seed(H + C)
    x = torch.randn(n, H, C, generator=g)
    att_s = torch.randn(1, H, C, generator=g)
    att_d = torch.randn(1, H, C, generator=g)
    gs, gd = torch.randn(n, H, generator=g), torch.randn(n, H, generator=g)
    leaves = [t.clone().requires_grad_(True) for t in (x, att_s, att_d)]
    a_s, a_d = ops.attention_logits(*leaves)
    go = torch.autograd.grad((a_s * gs).sum() + (a_d * gd).sum(), leaves)
    lg = [t.to(cuda).requires_grad_(True) for t in (x, att_s, att_d)]
    b_s, b_d = fused_attention_logits(*lg)
    ((b_s * gs.to(cuda)).sum() + (b_d * gd.to(cuda)).sum()).backward()
    assert_parity(b_s, a_s.detach(), what="alpha_src")
    assert_parity(b_d, a_d.detach(), what="alpha_dst")
    for t, e, name in zip(lg, go, ("grad_x", "grad_att_src", "grad_att_dst")):
        assert_parity(t.grad, e, what=name)
    # head mean + bias + SiLU
    out = torch.randn(n, H, C, generator=g)
    bias = torch.randn(C, generator=g)
    gy = torch.randn(n, C, generator=g)
    lo = [out.clone().requires_grad_(True), bias.clone().requires_grad_(True)]
    yo = ops.head_mean_bias_silu(*lo)
    go2 = torch.autograd.grad(yo, lo, gy)
    lgo = [out.to(cuda).requires_grad_(True), bias.to(cuda).requires_grad_(True)]
    y = fused_head_mean_bias_silu(*lgo)
    y.backward(gy.to(cuda))
    assert_parity(y, yo.detach(), what="head silu")
    assert_parity(lgo[0].grad, go2[0], what="head silu grad out")
    assert_parity(lgo[1].grad, go2[1], what="head silu grad bias")


def test_gat_deterministic(cuda):
    n, H, C = 800, 4, 128
    edge = prepare_gat_edge_index(synth.powerlaw_graph(n, 8000, seed=2), n)
    gpu_graph, _ = _graph(edge, n, cuda)
    plan = gat_plan_for(gpu_graph[0][0], gpu_graph[0][1], gpu_graph[1][0], gpu_graph[1][1],
                        gpu_graph[2])
    x = torch.randn(n, H, C, device=cuda)
    a = torch.randn(n, H, device=cuda)
    b = torch.zeros(C, device=cuda)
    gy = torch.randn(n, C, device=cuda)
    r1 = collapsed_gat.gat_forward_raw(plan, a, a, x, b, 0.2, 0.5, 99)
    g1 = collapsed_gat.gat_backward_raw(plan, a, a, x, r1[1], r1[2], r1[3], gy, 0.2, 0.5, 99)
    r2 = collapsed_gat.gat_forward_raw(plan, a, a, x, b, 0.2, 0.5, 99)
    g2 = collapsed_gat.gat_backward_raw(plan, a, a, x, r2[1], r2[2], r2[3], gy, 0.2, 0.5, 99)
    for u, v in zip(r1 + g1, r2 + g2):
        assert torch.equal(u, v)
