"""The tcgen05 pack + proj GEMM (cign_pack_proj_gemm_tf32) against the pack
kernel followed by a float64 matmul.

Two references per case:
  * the kernel's own G and W rounded to TF32 (round to nearest, ties away
    from zero -- what it feeds the tensor core) and multiplied in float64:
    the kernel may differ only by its fp32 accumulation order (1e-5
    relative);
  * the exact fp32 operands in float64: the TF32 contraction tolerance of
    2e-3 relative to the output's scale.
The optional G output must match the pack kernel's output (1e-5 relative:
the kernel's SiLU uses the hardware exponential).  Every call's
device status word is checked (no bounded wait expired)."""
import pytest
import torch

from cign_b200 import _pack
from tests.helpers import rel_l2

pytestmark = pytest.mark.gpu

MODES = (1, 0, 0)  # interaction "new", outer none, weighting "old"


def tf32_rna(x: torch.Tensor) -> torch.Tensor:
    """fp32 -> TF32 (10 explicit mantissa bits), round half away from zero."""
    bits = x.contiguous().view(torch.int32)
    return ((bits + 0x1000) & ~0x1FFF).view(torch.float32)


def make_case(n, D, K, dout, seed, device):
    g = torch.Generator(device="cpu").manual_seed(seed)
    H = torch.randn(n, D, generator=g).to(device)
    C = torch.randn(n, D, generator=g).to(device)
    props = [torch.randn(n, 2 * D, generator=g).to(device) for _ in range(K)]
    alpha = torch.softmax(torch.randn(n, K, generator=g), 1).to(device)
    W = (torch.randn(dout, 2 * K * D, generator=g) / (2 * K * D) ** 0.5).to(device)
    b = torch.randn(dout, generator=g).to(device)
    return H, C, props, alpha, W, b


@pytest.mark.parametrize("n,D,K,dout", [(300, 64, 3, 64), (1000, 32, 1, 32),
                                        (777, 128, 2, 256), (2000, 512, 3, 512),
                                        (129, 96, 4, 160)])
def test_pack_proj_matches_pack_then_matmul(cuda, n, D, K, dout):
    H, C, props, alpha, W, b = make_case(n, D, K, dout, seed=n + D + K + dout, device=cuda)
    out, G, ws = _pack.pack_proj_call(H, C, props, alpha, W, b, keep_g=True)
    _pack.pack_proj_status(ws, D, K, dout)
    G_ref = _pack.pack_forward(H, C, props, alpha, *MODES)
    # the kernel's SiLU uses the hardware exponential (~1e-6 relative)
    torch.testing.assert_close(G, G_ref, rtol=1e-5, atol=1e-6)

    emulated = tf32_rna(G).double() @ tf32_rna(W).double().t() + b.double()
    assert rel_l2(out, emulated) <= 1e-5, rel_l2(out, emulated)
    exact = G_ref.double() @ W.double().t() + b.double()
    scale = float(exact.abs().max())
    err = float((out.double() - exact).abs().max())
    assert err <= 2e-3 * scale, (err, scale)

    out2, G2 = _pack.pack_proj_forward(H, C, props, alpha, W, b, keep_g=False)
    assert G2 is None
    assert torch.equal(out, out2)  # deterministic, G output or not


def test_pack_proj_zero_rows(cuda):
    H, C, props, alpha, W, b = make_case(0, 64, 2, 64, seed=1, device=cuda)
    out, G, ws = _pack.pack_proj_call(H, C, props, alpha, W, b, keep_g=True)
    _pack.pack_proj_status(ws, 64, 2, 64)
    assert out.shape == (0, 64) and G.shape == (0, 256)


def test_pack_proj_rejects_unsupported(cuda):
    H, C, props, alpha, W, b = make_case(64, 48, 2, 64, seed=2, device=cuda)
    with pytest.raises(RuntimeError, match="multiple of 32"):
        _pack.pack_proj_call(H, C, props, alpha, W, b, keep_g=False)
