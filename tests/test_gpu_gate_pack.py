"""The hop gate evaluated inside the pack forward (cign_gate_pack_fwd)
against the two kernels it replaces, cign_hop_gate_fwd followed by
cign_pack_fwd: alpha and the packed output bit for bit, both gate score
modes and both weighting modes, every hop count 1..8 at a few widths, and
against the reference's torch hop gate and the oracle's pack (1e-5
relative)."""
import pytest
import torch
import torch.nn.functional as F

from cign_b200 import _pack
from cign_b200.hop_gate import hop_gate_forward_raw
from oracle import ops
from tests.helpers import assert_parity

pytestmark = pytest.mark.gpu


def _case(n, D, K, seed, device):
    g = torch.Generator().manual_seed(seed)
    H = torch.randn(n, D, generator=g).to(device)
    C = torch.randn(n, D, generator=g).to(device)
    props = [torch.randn(n, 2 * D, generator=g).to(device) for _ in range(K)]
    W = (torch.randn(K, 2 * D, generator=g) / (2 * D) ** 0.5).to(device)
    b = torch.randn(K, generator=g).to(device)
    return H, C, props, W, b


@pytest.mark.parametrize("D", [4, 96, 512, 1024])
@pytest.mark.parametrize("K", [1, 2, 3, 5, 8])
@pytest.mark.parametrize("gate_mode,interaction,outer,weighting",
                         [(1, 1, 0, 0), (0, 0, 1, 1), (1, 1, 1, 1)])
def test_gate_pack_equals_gate_then_pack(cuda, D, K, gate_mode, interaction, outer, weighting):
    H, C, props, W, b = _case(333, D, K, seed=D * 17 + K, device=cuda)
    assert _pack.gate_pack_supported(H, C, props)
    G, alpha = _pack.gate_pack_forward(H, C, props, W, b, gate_mode, interaction, outer, weighting)
    alpha_ref = hop_gate_forward_raw(H, C, W, b, gate_mode)
    G_ref = _pack.pack_forward(H, C, props, alpha_ref, interaction, outer, weighting)
    assert torch.equal(alpha, alpha_ref)
    assert torch.equal(G, G_ref)


def test_gate_pack_vs_oracle(cuda):
    n, D, K = 1000, 512, 3
    H, C, props, W, b = _case(n, D, K, seed=5, device=cuda)
    G, alpha = _pack.gate_pack_forward(H, C, props, W, b, 1, 1, 0, 0)
    Hc, Cc = H.cpu(), C.cpu()
    gate = torch.cat([Hc + Cc, torch.abs(Hc - Cc)], -1)  # model_cign.py:733-749
    a_ref = F.softmax(F.linear(gate, W.cpu(), b.cpu()), dim=-1)
    G_ref = ops.pack(Hc, Cc, [p.cpu() for p in props], a_ref, "new", "none", "old")
    assert_parity(alpha, a_ref, what="alpha")
    assert_parity(G, G_ref, what="G")


def test_gate_pack_edges(cuda):
    H, C, props, W, b = _case(0, 64, 2, seed=1, device=cuda)
    G, alpha = _pack.gate_pack_forward(H, C, props, W, b, 1, 1, 0, 0)
    assert G.shape == (0, 256) and alpha.shape == (0, 2)
    H, C, props, W, b = _case(8, 1028, 2, seed=2, device=cuda)
    assert not _pack.gate_pack_supported(H, C, props)
    with pytest.raises(RuntimeError, match="D <= 1024"):
        _pack.gate_pack_forward(H, C, props, W, b, 1, 1, 0, 0)
    H, C, props, W, b = _case(8, 64, 2, seed=3, device=cuda)
    props[1] = torch.randn(8 * 2 * 64 + 1, device=cuda)[1:].view(8, 128)
    assert not _pack.gate_pack_supported(H, C, props)
