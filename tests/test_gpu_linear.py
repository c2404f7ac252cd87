"""cign_b200.linear (fixed-order bias-gradient column sums, row-split weight
gradient for narrow inputs) against torch's F.linear autograd, fp32."""
import pytest
import torch
import torch.nn.functional as F

from cign_b200.linear import colsum, linear
from tests.helpers import assert_parity

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,k,m", [(1000, 300, 512), (20000, 300, 512), (24492, 3072, 512),
                                   (17, 5, 3)])
def test_linear_matches_torch(cuda, n, k, m):
    g = torch.Generator().manual_seed(n + k)
    x = torch.randn(n, k, generator=g)
    w = torch.randn(m, k, generator=g) / k ** 0.5
    b = torch.randn(m, generator=g)
    gy = torch.randn(n, m, generator=g)
    ref_in = [t.to(cuda).requires_grad_(True) for t in (x, w, b)]
    ref = F.linear(*ref_in)
    ref_g = torch.autograd.grad(ref, ref_in, gy.to(cuda))
    ins = [t.to(cuda).requires_grad_(True) for t in (x, w, b)]
    out = linear(*ins)
    grads = torch.autograd.grad(out, ins, gy.to(cuda))
    assert_parity(out, ref.detach(), what=f"y {n}x{k}x{m}")
    for name, a, e in zip(("grad_x", "grad_w", "grad_b"), grads, ref_g):
        assert_parity(a, e, what=f"{name} {n}x{k}x{m}")


def test_colsum_deterministic(cuda):
    a = torch.randn(24492, 512, device=cuda)
    s1, s2 = colsum(a), colsum(a)
    assert torch.equal(s1, s2)
    assert_parity(s1, a.double().sum(0).float(), what="colsum")
