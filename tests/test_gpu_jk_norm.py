"""cign_jk_ln_fwd/bwd (the model's output LayerNorm over the block states,
read without concatenating them) against torch's layer_norm of the
concatenation: outputs, the per-state input gradients and the LayerNorm
weight/bias gradients (fp32 parity, 1e-5 relative)."""
import pytest
import torch
import torch.nn.functional as F

from cign_b200.jk_norm import jk_layer_norm
from tests.helpers import assert_parity

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,S,W", [(1000, 3, 512), (777, 2, 64), (33, 5, 100), (4096, 8, 256)])
def test_jk_layer_norm_matches_torch(cuda, n, S, W):
    g = torch.Generator(device="cpu").manual_seed(n + S + W)
    states = [(torch.randn(n, W, generator=g) * (1 + i) + i).to(cuda) for i in range(S)]
    w = (1 + 0.1 * torch.randn(S * W, generator=g)).to(cuda)
    b = (0.1 * torch.randn(S * W, generator=g)).to(cuda)
    gy = torch.randn(n, S * W, generator=g).to(cuda)

    xs = [s.clone().requires_grad_(True) for s in states]
    wa, ba = w.clone().requires_grad_(True), b.clone().requires_grad_(True)
    out = jk_layer_norm(xs, wa, ba, 1e-5)
    out.backward(gy)

    xr = [s.clone().requires_grad_(True) for s in states]
    wr, br = w.clone().requires_grad_(True), b.clone().requires_grad_(True)
    ref = F.layer_norm(torch.cat(xr, -1), (S * W,), wr, br, 1e-5)
    ref.backward(gy)

    assert_parity(out.detach(), ref.detach(), what="y")
    for i, (a, r) in enumerate(zip(xs, xr)):
        assert_parity(a.grad, r.grad, what=f"grad state {i}")
    assert_parity(wa.grad, wr.grad, what="grad weight")
    assert_parity(ba.grad, br.grad, what="grad bias")


def test_jk_layer_norm_rejects_wide_rows(cuda):
    states = [torch.zeros(8, 1028, device=cuda) for _ in range(2)]
    w = torch.ones(2056, device=cuda)
    with pytest.raises(ValueError):
        jk_layer_norm(states, w, w, 1e-5)
