"""The fused dual input projection (cign_b200.input_proj: one stacked GEMM +
cign_silu_mix_fwd/_bwd) against the reference's expression
SiLU(x W0^T + b0) + eta * SiLU(x W1^T + b1) (generic_engine/model_cign.py:
1162-1170) in float64: output and the gradients of W0, b0, W1, b1 and eta
within 1e-5 relative (rel-L2), TF32 off."""
import pytest
import torch
import torch.nn.functional as F

from cign_b200.input_proj import dual_input_projection, silu_mix_backward, silu_mix_forward
from tests.helpers import assert_parity

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,i,d", [(1000, 300, 512), (257, 12, 4), (64, 100, 132), (0, 8, 16)])
def test_dual_input_projection_vs_reference(cuda, n, i, d):
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        g = torch.Generator().manual_seed(n + i + d)
        x = torch.randn(n, i, generator=g)
        w0 = torch.randn(d, i, generator=g) / i ** 0.5
        w1 = torch.randn(d, i, generator=g) / i ** 0.5
        b0 = torch.randn(d, generator=g) * 0.1
        b1 = torch.randn(d, generator=g) * 0.1
        eta = torch.tensor(0.37)
        gy = torch.randn(n, d, generator=g)
        ref_leaves = [t.double().requires_grad_(True) for t in (w0, b0, w1, b1, eta)]
        xd = x.double()
        ref = (F.silu(F.linear(xd, ref_leaves[0], ref_leaves[1]))
               + ref_leaves[4] * F.silu(F.linear(xd, ref_leaves[2], ref_leaves[3])))
        ref_grads = torch.autograd.grad(ref, ref_leaves, gy.double()) if n else None
        leaves = [t.to(cuda).requires_grad_(True) for t in (w0, b0, w1, b1, eta)]
        y = dual_input_projection(x.to(cuda), *leaves[:4], leaves[4])
        assert y.shape == (n, d)
        if n == 0:
            return
        assert_parity(y, ref.detach().float(), what="H")
        grads = torch.autograd.grad(y, leaves, gy.to(cuda))
        for name, a, e in zip(("w0", "b0", "w1", "b1", "eta"), grads, ref_grads):
            assert_parity(a, e.float(), what=f"grad {name}")
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def test_silu_mix_deterministic(cuda):
    g = torch.Generator().manual_seed(3)
    z = torch.randn(24492, 1024, generator=g).to(cuda)
    gy = torch.randn(24492, 512, generator=g).to(cuda)
    eta = torch.tensor([0.1], device=cuda)
    a = silu_mix_forward(z, eta)
    assert torch.equal(a, silu_mix_forward(z, eta))
    gz1, ge1 = silu_mix_backward(gy, z, eta)
    gz2, ge2 = silu_mix_backward(gy, z, eta)
    assert torch.equal(gz1, gz2) and torch.equal(ge1, ge2)
