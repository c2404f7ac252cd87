"""The CPU oracle against outputs of the REFERENCE's own CUDA kernels
(tests/golden/ref_gat_family.npz and ref_block_ops_gpu.npz, written on a
B200 by tests/golden/make_ref_gpu_golden.py from the reference's unchanged
collapsed_gat_ext, fused_gat_sideops_ext and fused_block_ops_ext sources).
This pins the GAT-family and block-op restatements of oracle/ to the
reference itself.  CPU only.

The reference's [nnz,H] mask is left unwritten when attn_drop is 0
(collapsed_gat_cuda.cu:462-470 launches the mask kernel only for p > 0, and
the aggregation never reads it then), so masks are compared at p = 0.5 only.
"""
import numpy as np
import pytest
import torch

from oracle import ops, rng
from tests.helpers import assert_parity


def _t(z, k):
    return torch.from_numpy(np.ascontiguousarray(z[k]))


@pytest.fixture(scope="module")
def gat(golden):
    return golden("ref_gat_family.npz")


@pytest.mark.parametrize("tag,p", [("p0", 0.0), ("p50", 0.5)])
def test_collapsed_gat_oracle_vs_reference_kernel(gat, tag, p):
    z = gat
    seed = int(z["seed_p50"]) if p > 0 else 0
    leaves = [_t(z, k).clone().requires_grad_(True)
              for k in ("attn_row", "attn_col", "in_feat", "bias")]
    out, pre, emax, esum = ops.gat_collapsed(leaves[0], leaves[1], z["rowptr"], z["col"], leaves[2],
                                             leaves[3], float(z["negative_slope"]), p, seed)
    grads = torch.autograd.grad(out, leaves, _t(z, "grad_y"))
    assert_parity(out.detach(), _t(z, f"out_{tag}"), what=f"out {tag}")
    assert_parity(pre.detach(), _t(z, f"pre_{tag}"), what=f"pre {tag}")
    assert_parity(emax, _t(z, f"edge_max_{tag}"), what=f"edge_max {tag}")
    assert_parity(esum, _t(z, f"edge_sum_{tag}"), what=f"edge_sum {tag}")
    for name, g in zip(("grad_attn_row", "grad_attn_col", "grad_feat", "grad_bias"), grads):
        assert_parity(g, _t(z, f"{name}_{tag}"), what=f"{name} {tag}")


def test_gat_dropout_mask_oracle_vs_reference_kernel(gat):
    z = gat
    nnz, H = z["edge_mask_p50"].shape
    keep = rng.gat_keep_mask(int(z["seed_p50"]), nnz * H, 0.5).reshape(nnz, H)
    np.testing.assert_array_equal(keep.astype(np.uint8), z["edge_mask_p50"])


def test_attention_logits_oracle_vs_reference_kernel(gat):
    z = gat
    x = _t(z, "in_feat").clone().requires_grad_(True)
    a_s = _t(z, "att_src").clone().requires_grad_(True)
    a_d = _t(z, "att_dst").clone().requires_grad_(True)
    src, dst = ops.attention_logits(x, a_s, a_d)
    assert_parity(src.detach(), _t(z, "alpha_src"), what="alpha_src")
    assert_parity(dst.detach(), _t(z, "alpha_dst"), what="alpha_dst")
    gx, gs, gd = torch.autograd.grad((src, dst), (x, a_s, a_d), (_t(z, "grad_src"), _t(z, "grad_dst")))
    assert_parity(gx, _t(z, "logits_grad_x"), what="grad_x")
    assert_parity(gs, _t(z, "logits_grad_att_src"), what="grad_att_src")
    assert_parity(gd, _t(z, "logits_grad_att_dst"), what="grad_att_dst")


def test_head_mean_bias_silu_oracle_vs_reference_kernel(gat):
    z = gat
    x = _t(z, "in_feat").clone().requires_grad_(True)
    b = _t(z, "bias").clone().requires_grad_(True)
    y = ops.head_mean_bias_silu(x, b)
    assert_parity(y.detach(), _t(z, "head_y"), what="head y")
    assert_parity(x.detach().mean(1) + b.detach(), _t(z, "head_pre"), what="head pre")
    gx, gb = torch.autograd.grad(y, (x, b), _t(z, "grad_y"))
    assert_parity(gx, _t(z, "head_grad_out"), what="head grad_out")
    assert_parity(gb, _t(z, "head_grad_bias"), what="head grad_bias")


@pytest.mark.parametrize("D", [256, 96])
def test_block_ops_oracle_vs_reference_kernels(golden, D):
    z = golden("ref_block_ops_gpu.npz")
    pre = f"d{D}_"
    p, eps = float(z["p"]), float(z["eps"])
    ln_seed, gamma_seed = int(z["ln_seed"]), int(z["gamma_seed"])
    n = z[pre + "x"].shape[0]

    # masks: bit for bit
    np.testing.assert_array_equal(
        rng.block_keep_mask(ln_seed, n * D, p).reshape(n, D).astype(np.uint8), z[pre + "dln_mask"])
    np.testing.assert_array_equal(
        rng.block_keep_mask(gamma_seed, n * D, p).reshape(n, D).astype(np.uint8),
        z[pre + "gres_mask"])

    def leaf(k):
        return _t(z, pre + k).clone().requires_grad_(True)

    gy = _t(z, pre + "gy")
    # dropout + LayerNorm
    x, w, b = leaf("x"), leaf("w"), leaf("bb")
    y = ops.dropout_layernorm(x, w, b, p, eps, ln_seed)
    assert_parity(y.detach(), _t(z, pre + "dln_y"), what=f"dropout-LN y D={D}")
    q = ops._block_dropout(x.detach(), p, ln_seed)
    assert_parity(q.mean(1), _t(z, pre + "dln_mean"), atol=1e-6, what="dropout-LN mean")
    rstd = torch.rsqrt(q.var(1, unbiased=False) + eps)
    assert_parity(rstd, _t(z, pre + "dln_rstd"), what="dropout-LN rstd")
    for name, g in zip(("dln_dx", "dln_gw", "dln_gb"), torch.autograd.grad(y, (x, w, b), gy)):
        assert_parity(g, _t(z, pre + name), what=f"{name} D={D}")
    # add + LayerNorm
    a, bb = leaf("a"), leaf("b")
    w2, b2 = leaf("w"), leaf("bb")
    y = ops.add_layernorm(a, bb, w2, b2, eps)
    assert_parity(y.detach(), _t(z, pre + "aln_y"), what=f"add-LN y D={D}")
    ga, gbb, gw, gb = torch.autograd.grad(y, (a, bb, w2, b2), gy)
    assert_parity(ga, _t(z, pre + "aln_dz"), what=f"add-LN dz D={D}")
    assert_parity(gbb, _t(z, pre + "aln_dz"), what=f"add-LN dz (b) D={D}")
    assert_parity(gw, _t(z, pre + "aln_gw"), what=f"add-LN gw D={D}")
    assert_parity(gb, _t(z, pre + "aln_gb"), what=f"add-LN gb D={D}")
    # dropout-gamma-residual
    h, g, gamma = leaf("h"), leaf("gm"), leaf("gamma")
    y = ops.dropout_gamma_residual(h, g, gamma, p, gamma_seed)
    assert_parity(y.detach(), _t(z, pre + "gres_y"), what=f"gamma-res y D={D}")
    _, gg, ggamma = torch.autograd.grad(y, (h, g, gamma), gy)
    assert_parity(gg, _t(z, pre + "gres_gg"), what=f"gamma-res grad_g D={D}")
    assert_parity(ggamma, _t(z, pre + "gres_ggamma"), what=f"gamma-res grad_gamma D={D}")
