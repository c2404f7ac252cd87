"""Fused hop gate (cign_hop_gate_fwd/_bwd) vs the reference's torch
expression (generic_engine/model_cign.py:733-749) in fp32 on the CPU:
softmax(Linear(cat[H+C, |H-C|])) ("new") and softmax(Linear(cat[H, C]))
("old"), forward and the gradients of H, C, weight and bias."""
import pytest
import torch
import torch.nn.functional as F

from cign_b200.hop_gate import fused_hop_gate
from tests.helpers import assert_parity

pytestmark = pytest.mark.gpu


def _reference(h, c, w, b, mode):
    gate = torch.cat([h, c], -1) if mode == "old" else torch.cat([h + c, torch.abs(h - c)], -1)
    return F.softmax(F.linear(gate, w, b), dim=-1)


@pytest.mark.parametrize("n,d,k", [(1000, 512, 3), (257, 4, 1), (300, 132, 8), (64, 64, 5)])
@pytest.mark.parametrize("mode", ["new", "old"])
def test_hop_gate_vs_torch(cuda, n, d, k, mode):
    g = torch.Generator().manual_seed(n + d + k)
    h = torch.randn(n, d, generator=g)
    c = torch.randn(n, d, generator=g)
    c[: n // 10] = h[: n // 10]  # |H - C| at 0: sign(0) = 0 in the backward
    w = torch.randn(k, 2 * d, generator=g) / (2 * d) ** 0.5
    b = torch.randn(k, generator=g)
    ga = torch.randn(n, k, generator=g)
    leaves = [t.clone().requires_grad_(True) for t in (h, c, w, b)]
    ref = _reference(*leaves, mode)
    grads_ref = torch.autograd.grad(ref, leaves, ga)
    ins = [t.to(cuda).requires_grad_(True) for t in (h, c, w, b)]
    out = fused_hop_gate(*ins, score_mode=mode)
    grads = torch.autograd.grad(out, ins, ga.to(cuda))
    tag = f"n={n} d={d} k={k} {mode}"
    assert_parity(out, ref.detach(), what=f"alpha {tag}")
    for name, a, e in zip(("grad_h", "grad_c", "grad_w", "grad_b"), grads, grads_ref):
        assert_parity(a, e, what=f"{name} {tag}")


def test_hop_gate_deterministic(cuda):
    g = torch.Generator(device=cuda).manual_seed(0)
    h, c = torch.randn(24492, 512, device=cuda, generator=g), torch.randn(24492, 512, device=cuda, generator=g)
    w = torch.randn(3, 1024, device=cuda, generator=g, requires_grad=True)
    b = torch.zeros(3, device=cuda, requires_grad=True)
    ga = torch.randn(24492, 3, device=cuda, generator=g)
    r1 = torch.autograd.grad(fused_hop_gate(h, c, w, b), (w, b), ga)
    r2 = torch.autograd.grad(fused_hop_gate(h, c, w, b), (w, b), ga)
    assert all(torch.equal(x, y) for x, y in zip(r1, r2))
