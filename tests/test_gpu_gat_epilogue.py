"""The GAT epilogue fused with the block's add-LayerNorm
(gat_silu_add_layernorm: LN(SiLU(lin + bias) + h)) against the torch fp32
expression of the reference's unfused ops (model_cign.py:767-787:
SiLU(GAT + bias), then LayerNorm(C + H_norm)), forward and every gradient,
and against this library's op-by-op path (head-mean-bias-SiLU, then add-LN)."""
import pytest
import torch
import torch.nn.functional as F

from cign_b200.collapsed_gat import _bias_silu, gat_silu_add_layernorm, silu_add_ln_forward
from cign_b200.fused_block_ops import add_ln_forward
from tests.helpers import assert_parity

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,D", [(777, 512), (1001, 24), (300, 100), (64, 1024), (0, 64)])
def test_silu_add_layernorm_vs_torch(cuda, n, D):
    g = torch.Generator().manual_seed(n + D)
    lin, h, gy = (torch.randn(n, D, generator=g) for _ in range(3))
    bias = 0.3 * torch.randn(D, generator=g)
    w = 1.0 + 0.1 * torch.randn(D, generator=g)
    b = 0.1 * torch.randn(D, generator=g)
    eps = 1e-5
    leaves = [t.clone().requires_grad_(True) for t in (lin, bias, h, w, b)]
    ref = F.layer_norm(F.silu(leaves[0] + leaves[1]) + leaves[2], (D,), leaves[3], leaves[4], eps)
    ref_grads = torch.autograd.grad(ref, leaves, gy) if n else [torch.zeros_like(t) for t in leaves]
    dev = [t.to(cuda).requires_grad_(True) for t in (lin, bias, h, w, b)]
    y = gat_silu_add_layernorm(*dev, eps)
    y.backward(gy.to(cuda))
    if n == 0:
        assert y.shape == (0, D)
        for t in dev[1:2] + dev[3:]:
            assert bool((t.grad == 0).all())
        return
    assert_parity(y, ref.detach(), what=f"y n={n} D={D}")
    for name, t, e in zip(("lin", "bias", "h", "ln_w", "ln_b"), dev, ref_grads):
        assert_parity(t.grad, e, what=f"grad {name} n={n} D={D}")


def test_silu_add_layernorm_forward_equals_op_by_op(cuda):
    """The same formulas as the two separate kernels: pre bit for bit, the
    rest within 1e-6 (the fused pass may round SiLU(pre) + h as one FMA
    where the separate kernels round SiLU(pre) first)."""
    n, D = 2048, 512
    g = torch.Generator(device=cuda).manual_seed(3)
    lin, h = torch.randn(n, D, device=cuda, generator=g), torch.randn(n, D, device=cuda, generator=g)
    bias = torch.randn(D, device=cuda, generator=g)
    w, b = torch.randn(D, device=cuda, generator=g), torch.randn(D, device=cuda, generator=g)
    y, pre, mean, rstd = silu_add_ln_forward(lin, bias, h, w, b, 1e-5)
    c, pre2 = _bias_silu(lin, bias)
    y2, mean2, rstd2 = add_ln_forward(c, h, w, b, 1e-5)
    assert torch.equal(pre, pre2)
    for name, a, e in (("y", y, y2), ("mean", mean, mean2), ("rstd", rstd, rstd2)):
        assert_parity(a, e, tol=1e-6, what=name)
