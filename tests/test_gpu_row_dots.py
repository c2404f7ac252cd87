"""Row dots (cign_row_dots_fwd/_bwd) against float64, and the GAT context
node that uses them for its attention logits (collapsed_gat.gat_context:
lin(x) -> logits -> collapsed GAT -> bias + SiLU in one node) against the
CPU oracle of the reference order: in_feat = lin(x).view(N, H, C), the
logits of fused_gat_sideops.py:50-71 on in_feat, the collapsed GAT
(collapsed_gat_cuda.cu:52-545 restated in oracle.ops).  fp32 within 1e-5
relative (rel-L2)."""
import pytest
import torch

from cign_b200 import collapsed_gat, synth
from cign_b200.collapsed_gat import gat_context, row_dots_backward, row_dots_forward
from cign_b200.graph_operator import prepare_gat_edge_index, to_graph_format
from oracle import ops
from tests.helpers import assert_parity

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,D,K", [(1000, 512, 8), (257, 4, 1), (300, 132, 16), (64, 64, 3),
                                   (0, 64, 4)])
@pytest.mark.parametrize("accumulate", [False, True])
def test_row_dots_vs_float64(cuda, n, D, K, accumulate):
    g = torch.Generator().manual_seed(n + D + K)
    x = torch.randn(n, D, generator=g)
    V = torch.randn(K, D, generator=g) / D ** 0.5
    go = torch.randn(n, K, generator=g)
    base = torch.randn(n, D, generator=g)
    out = row_dots_forward(x.to(cuda), V.to(cuda))
    assert out.shape == (n, K)
    if n:
        assert_parity(out, (x.double() @ V.double().t()).float(), what="row dots")
    gx = base.to(cuda).clone() if accumulate else torch.empty(n, D, device=cuda)
    gV = row_dots_backward(x.to(cuda), V.to(cuda), go.to(cuda), gx, accumulate)
    want_gx = go.double() @ V.double() + (base.double() if accumulate else 0)
    want_gV = go.double().t() @ x.double()
    if n:
        assert_parity(gx, want_gx.float(), what="grad_x")
        assert_parity(gV, want_gV.float(), what="grad_V")
    else:
        assert torch.count_nonzero(gV) == 0


def test_row_dots_deterministic(cuda):
    g = torch.Generator().manual_seed(3)
    x = torch.randn(24492, 512, generator=g).to(cuda)
    V = torch.randn(8, 512, generator=g).to(cuda)
    go = torch.randn(24492, 8, generator=g).to(cuda)
    gx1, gx2 = torch.empty_like(x), torch.empty_like(x)
    gV1 = row_dots_backward(x, V, go, gx1, False)
    gV2 = row_dots_backward(x, V, go, gx2, False)
    assert torch.equal(gV1, gV2) and torch.equal(gx1, gx2)


def _oracle_context(x, W, att_src, att_dst, bias, rp, c, H, C, slope, p, seed):
    xh = (x @ W.t()).view(-1, H, C)
    a_src, a_dst = ops.attention_logits(xh, att_src, att_dst)
    out, _, _, _ = ops.gat_collapsed(a_dst, a_src, rp, c, xh, bias, slope, p, seed)
    return out


@pytest.mark.parametrize("H,D,C,p", [(4, 64, 64, 0.0), (2, 32, 16, 0.5), (1, 128, 128, 0.3)])
def test_gat_context_vs_reference_order(cuda, monkeypatch, H, D, C, p):
    n = 600
    edge = prepare_gat_edge_index(synth.powerlaw_graph(n, 5000, seed=H + D), n)
    (rp, c), (r, cp), perm = to_graph_format(edge.flip(0), n)
    g = torch.Generator().manual_seed(7 * H + D)
    x = torch.randn(n, D, generator=g)
    W = torch.randn(H * C, D, generator=g) / D ** 0.5
    att_src = torch.randn(1, H, C, generator=g) / C ** 0.5
    att_dst = torch.randn(1, H, C, generator=g) / C ** 0.5
    bias = torch.randn(C, generator=g) * 0.1
    gy = torch.randn(n, C, generator=g)
    seed = 12345 if p > 0 else 0
    leaves = [t.clone().requires_grad_(True) for t in (x, W, att_src, att_dst, bias)]
    out_o = _oracle_context(*leaves, rp, c, H, C, 0.2, p, seed)
    grads_o = torch.autograd.grad(out_o, leaves, gy)

    ins = [t.to(cuda).requires_grad_(True) for t in (x, W, att_src, att_dst, bias)]
    dev = lambda t: t.to(cuda)  # noqa: E731
    monkeypatch.setattr(collapsed_gat, "gat_call_seed", lambda attn_drop: seed)
    out = gat_context(ins[0], ins[1], ins[2], ins[3], ins[4], (dev(rp), dev(c)),
                      (dev(r), dev(cp)), dev(perm), 0.2, p)
    grads = torch.autograd.grad(out, ins, gy.to(cuda))
    tag = f"H={H} D={D} C={C} p={p}"
    assert_parity(out, out_o.detach(), what=f"out {tag}")
    for name, a, e in zip(("grad_x", "grad_weight", "grad_att_src", "grad_att_dst", "grad_bias"),
                          grads, grads_o):
        assert_parity(a, e, what=f"{name} {tag}")
