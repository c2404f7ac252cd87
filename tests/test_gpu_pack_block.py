"""Clifford pack family and block side ops on the GPU vs the reference's
outputs (golden) and the CPU oracle (dropout masks bit for bit)."""
import numpy as np
import pytest
import torch

from cign_b200 import fused_block_ops as fbo
from cign_b200 import fused_clifford_cign_generic, fused_clifford_cign_pack, fused_clifford_pack
from cign_b200 import fused_clifford_switch_pack
from oracle import ops, rng
from tests.helpers import assert_parity

pytestmark = pytest.mark.gpu


def _api_call(kind, k, w, H, C, P, A):
    if kind == "cign":
        if k == 3:
            return fused_clifford_cign_pack.fused_clifford_switch_pack(H, C, P, A, "new", w)
        out = fused_clifford_cign_generic.fused_clifford_pack(H, C, P, A)
        if w == "new":
            n, d = H.shape
            packed = out.reshape(n, k, 2 * d)
            out = torch.cat([packed[..., d:].sum(1), packed[..., :d].sum(1)], dim=-1)
        return out
    if kind == "legacy":
        return fused_clifford_pack.fused_clifford_pack(H, C, P, A)
    inter = kind.split("_")[1]
    return fused_clifford_switch_pack.fused_clifford_switch_pack(H, C, P, A, inter, w)


def test_pack_golden(cuda, golden):
    z = golden("pack_cases.npz")
    for case in z["cases"]:
        tag, kind, k, d, w = str(case).split("|")
        k = int(k)
        leaves = [torch.from_numpy(z[f"{tag}_in{j}"]).to(cuda).requires_grad_(True)
                  for j in range(k + 3)]
        alpha = torch.softmax(leaves[-1], -1)
        y = _api_call(kind, k, w, leaves[0], leaves[1], leaves[2:-1], alpha)
        assert_parity(y.detach(), z[f"{tag}_y"], what=str(case))
        grads = torch.autograd.grad(y, leaves, torch.from_numpy(z[f"{tag}_go"]).to(cuda))
        for j, g in enumerate(grads):
            assert_parity(g, z[f"{tag}_g{j}"], what=f"{case} grad {j}")


@pytest.mark.parametrize("inter,outer,weight", [("new", "none", "old"), ("new", "none", "new"),
                                                ("old", "none", "old"), ("new", "tanh", "new")])
@pytest.mark.parametrize("K,D", [(3, 512), (2, 512), (8, 64), (1, 30), (5, 1024)])
def test_pack_large_vs_oracle(cuda, inter, outer, weight, K, D):
    from cign_b200._pack import run_pack
    n = 333
    g = torch.Generator().manual_seed(K * 1000 + D)
    raw = [torch.randn(n, D, generator=g), torch.randn(n, D, generator=g)] + \
        [torch.randn(n, 2 * D, generator=g) for _ in range(K)] + [torch.randn(n, K, 1, generator=g)]
    lo = [t.clone().requires_grad_(True) for t in raw]
    yo = ops.pack(lo[0], lo[1], lo[2:-1], torch.softmax(lo[-1], 1), inter, outer, weight)
    go = torch.randn(yo.shape, generator=g)
    gro = torch.autograd.grad(yo, lo, go)
    lg = [t.to(cuda).requires_grad_(True) for t in raw]
    y = run_pack(lg[0], lg[1], lg[2:-1], torch.softmax(lg[-1], 1), 0 if inter == "old" else 1,
                 1 if outer == "tanh" else 0, 0 if weight == "old" else 1)
    assert_parity(y.detach(), yo.detach(), what="pack fwd")
    grg = torch.autograd.grad(y, lg, go.to(cuda))
    for j, (a, e) in enumerate(zip(grg, gro)):
        assert_parity(a, e, what=f"pack grad {j}")


def test_pack_alpha_none(cuda):
    n, D, K = 50, 16, 3
    H, C = torch.randn(n, D), torch.randn(n, D)
    P = [torch.randn(n, 2 * D) for _ in range(K)]
    y = fused_clifford_cign_generic.fused_clifford_pack(H.to(cuda), C.to(cuda), [p.to(cuda) for p in P],
                                                       None)
    assert_parity(y, ops.pack(H, C, P, None, "new", "none", "old"), what="alpha None")


def test_block_ops_golden(cuda, golden):
    z = golden("block_ops.npz")
    leaves = [torch.from_numpy(z[f"in{i}"]).to(cuda).requires_grad_(True) for i in range(8)]
    H, Cg, G, hw, hb, cw, cb, gamma = leaves
    Hn = fbo.fused_dropout_layernorm(H, hw, hb, 0.0, 1e-5)
    Cn = fbo.fused_add_layernorm(Cg, Hn, cw, cb, 1e-5)
    Y = fbo.fused_dropout_gamma_residual(H, G, gamma, 0.0)
    for name, t in (("Hn", Hn), ("Cn", Cn), ("Y", Y)):
        assert_parity(t.detach(), z[name], what=name)
    loss = sum((a * torch.from_numpy(z[f"go{i}"]).to(cuda)).sum() for i, a in enumerate((Hn, Cn, Y)))
    grads = torch.autograd.grad(loss, leaves)
    for i, g in enumerate(grads):
        assert_parity(g, z[f"g{i}"], what=f"block grad {i}")


@pytest.mark.parametrize("D", [24, 30, 48, 512, 1000, 1024])
@pytest.mark.parametrize("p", [0.0, 0.5])
def test_block_ops_vs_oracle(cuda, D, p):
    n = 700
    g = torch.Generator().manual_seed(D)
    x, a, gvec = torch.randn(n, D, generator=g), torch.randn(n, D, generator=g), torch.randn(n, D, generator=g)
    w, b = 1 + 0.1 * torch.randn(D, generator=g), 0.1 * torch.randn(D, generator=g)
    gamma = 0.49 + 0.05 * torch.randn(D, generator=g)
    gy = torch.randn(n, D, generator=g)
    seed_ln, seed_res = rng.block_seed(7, 1, 1), rng.block_seed(7, 2, 2)
    # dropout-LN
    lo = [t.clone().requires_grad_(True) for t in (x, w, b)]
    yo = ops.dropout_layernorm(lo[0], lo[1], lo[2], p, 1e-5, seed_ln)
    go = torch.autograd.grad(yo, lo, gy)
    lg = [t.to(cuda).requires_grad_(True) for t in (x, w, b)]
    y = fbo._DropoutLayerNormFn.apply(lg[0], lg[1], lg[2], p, 1e-5, seed_ln)
    y.backward(gy.to(cuda))
    assert_parity(y.detach(), yo.detach(), what=f"dropout_ln D={D}")
    for t, e, nm in zip(lg, go, ("x", "w", "b")):
        assert_parity(t.grad, e, tol=2e-5, what=f"dropout_ln grad {nm} D={D}")
    # add-LN
    lo = [t.clone().requires_grad_(True) for t in (x, a, w, b)]
    yo = ops.add_layernorm(*lo, 1e-5)
    go = torch.autograd.grad(yo, lo, gy)
    lg = [t.to(cuda).requires_grad_(True) for t in (x, a, w, b)]
    y = fbo.fused_add_layernorm(*lg, 1e-5)
    y.backward(gy.to(cuda))
    assert_parity(y.detach(), yo.detach(), what=f"add_ln D={D}")
    for t, e, nm in zip(lg, go, ("a", "b", "w", "bias")):
        assert_parity(t.grad, e, tol=2e-5, what=f"add_ln grad {nm} D={D}")
    # gamma residual
    lo = [t.clone().requires_grad_(True) for t in (x, gvec, gamma)]
    yo = ops.dropout_gamma_residual(lo[0], lo[1], lo[2], p, seed_res)
    go = torch.autograd.grad(yo, lo, gy)
    lg = [t.to(cuda).requires_grad_(True) for t in (x, gvec, gamma)]
    y = fbo._DropoutGammaResidualFn.apply(lg[0], lg[1], lg[2], p, seed_res)
    y.backward(gy.to(cuda))
    assert_parity(y.detach(), yo.detach(), what=f"gamma residual D={D}")
    for t, e, nm in zip(lg, go, ("h", "g", "gamma")):
        assert_parity(t.grad, e, what=f"gamma residual grad {nm} D={D}")


def test_block_mask_bit_exact_and_seed_stream(cuda):
    for seed, p in ((rng.block_seed(42, 1, 1), 0.28), (rng.block_seed(42, 9, 2), 0.5), (3, 0.9)):
        m = fbo.block_dropout_mask(100003, p, seed, cuda).cpu().numpy().astype(bool)
        np.testing.assert_array_equal(m, rng.block_keep_mask(seed, 100003, p))
    # module API: counter shared by both ops, advanced only for p > 0
    torch.manual_seed(42)
    call = next(fbo._CALL_COUNTER) + 1
    assert fbo._next_seed(1, 0.0) == 0
    assert fbo._next_seed(1, 0.3) == rng.block_seed(42, call + 1, 1)
    assert fbo._next_seed(2, 0.3) == rng.block_seed(42, call + 2, 2)
