"""The CPU oracle against the reference's own outputs (tests/golden/*.npz,
written by tests/golden/make_golden.py from the reference's Python code)
and against published known answers.  CPU only."""
import numpy as np
import pytest
import torch

from oracle import graph as og
from oracle import ops, rng
from oracle.model import OracleCIGN


def test_splitmix64_known_answers():
    # Published SplitMix64 outputs for state 0 (Vigna's splitmix64.c): the
    # finaliser applied to k * 0x9E3779B97F4A7C15, k = 0, 1, 2.
    g = 0x9E3779B97F4A7C15
    got = rng.splitmix64(np.array([0, g, (2 * g) % (1 << 64)], dtype=np.uint64))
    assert [int(v) for v in got] == [0xE220A8397B1DCDAF, 0x6E789E6AA1B965F4, 0x06C45D188009454F]


def test_mask_rates_and_seeds():
    m = rng.gat_keep_mask(12345, 200000, 0.3)
    assert abs(m.mean() - 0.7) < 0.01
    b = rng.block_keep_mask(999, 200000, 0.5)
    assert abs(b.mean() - 0.5) < 0.01
    assert rng.gat_keep_mask(5, 100, 0.0).all() and rng.block_keep_mask(5, 100, 0.0).all()
    # seed formulas (collapsed_gat.py:204-211, fused_block_ops.py:46-50)
    assert rng.gat_seed(42, 0) == (42 + 0x9E3779B97F4A7C15) & ((1 << 63) - 1)
    assert rng.block_seed(42, 1, 2) == (42 + 0x9E3779B97F4A7C15 + 2 * 0xD2B74407B1CE6E93) & ((1 << 63) - 1)


def test_fixed_csr_construction_bit_exact(golden):
    z = golden("fixedcsr_random.npz")
    n = int(z["n"])
    r, c, v = og.coalesce(z["coo_row"], z["coo_col"], z["coo_val"], n, n)
    crow, col, val = og.csr_of(r, c, v, n)
    np.testing.assert_array_equal(crow, z["crow"])
    np.testing.assert_array_equal(col, z["col"])
    np.testing.assert_allclose(val, z["val"], rtol=1e-6, atol=0)
    crow_t, col_t, val_t = og.csr_transpose(r, c, v, n)
    np.testing.assert_array_equal(crow_t, z["crow_t"])
    np.testing.assert_array_equal(col_t, z["col_t"])
    np.testing.assert_allclose(val_t, z["val_t"], rtol=1e-6, atol=0)


def test_fixed_spmm_fwd_bwd(golden):
    z = golden("fixedcsr_random.npz")
    n = int(z["n"])
    P = ops.csr_tensor(z["crow"], z["col"], z["val"], n, n)
    PT = ops.csr_tensor(z["crow_t"], z["col_t"], z["val_t"], n, n)
    x = torch.from_numpy(z["x"]).requires_grad_(True)
    y = ops.spmm(P, PT, x)
    (y * torch.from_numpy(z["gy"])).sum().backward()
    np.testing.assert_allclose(y.detach().numpy(), z["y"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(x.grad.numpy(), z["gx"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("name,powers", [("p123", (1, 2, 3)), ("p1248", (1, 2, 4, 8)),
                                         ("p0_2_5", (0, 2, 5))])
def test_multihop_fwd_bwd(golden, name, powers):
    z = golden("multihop_circulant.npz")
    n = int(z["n"])
    r, c, v = og.coalesce(z["coo_row"], z["coo_col"], z["coo_val"], n, n)
    P = ops.csr_tensor(*og.csr_of(r, c, v, n), n, n)
    PT = ops.csr_tensor(*og.csr_transpose(r, c, v, n), n, n)
    x = torch.from_numpy(z[f"{name}_x"]).requires_grad_(True)
    out = ops.multihop(P, PT, x, powers)
    loss = 0
    for p in powers:
        if p == 0:
            continue
        np.testing.assert_allclose(out[p].detach().numpy(), z[f"{name}_y{p}"], rtol=1e-5, atol=1e-6)
        loss = loss + (out[p] * torch.from_numpy(z[f"{name}_g{p}"])).sum()
    loss.backward()
    np.testing.assert_allclose(x.grad.numpy(), z[f"{name}_gx"], rtol=1e-5, atol=1e-6)


def _pack_modes(kind, w):
    if kind == "cign":
        return "new", "none", w
    if kind == "legacy":
        return "old", "none", "old"
    inter = kind.split("_")[1]
    return inter, "tanh", w


def test_pack_family(golden):
    z = golden("pack_cases.npz")
    for case in z["cases"]:
        tag, kind, k, d, w = str(case).split("|")
        k = int(k)
        inter, outer, weight = _pack_modes(kind, w)
        raw = [torch.from_numpy(z[f"{tag}_in{j}"]).requires_grad_(True) for j in range(k + 3)]
        alpha = torch.softmax(raw[-1], -1)
        y = ops.pack(raw[0], raw[1], raw[2:-1], alpha, inter, outer, weight)
        np.testing.assert_allclose(y.detach().numpy(), z[f"{tag}_y"], rtol=1e-5, atol=1e-6,
                                   err_msg=str(case))
        grads = torch.autograd.grad(y, raw, torch.from_numpy(z[f"{tag}_go"]))
        for j, g in enumerate(grads):
            np.testing.assert_allclose(g.numpy(), z[f"{tag}_g{j}"], rtol=1e-5, atol=1e-6,
                                       err_msg=f"{case} grad {j}")


def test_block_ops_p0(golden):
    z = golden("block_ops.npz")
    leaves = [torch.from_numpy(z[f"in{i}"]).requires_grad_(True) for i in range(8)]
    H, Cg, G, hw, hb, cw, cb, gamma = leaves
    Hn = ops.dropout_layernorm(H, hw, hb, 0.0, 1e-5, 0)
    Cn = ops.add_layernorm(Cg, Hn, cw, cb, 1e-5)
    Y = ops.dropout_gamma_residual(H, G, gamma, 0.0, 0)
    for name, t in (("Hn", Hn), ("Cn", Cn), ("Y", Y)):
        np.testing.assert_allclose(t.detach().numpy(), z[name], rtol=1e-5, atol=1e-6)
    loss = sum((a * torch.from_numpy(z[f"go{i}"])).sum() for i, a in enumerate((Hn, Cn, Y)))
    grads = torch.autograd.grad(loss, leaves)
    for i, g in enumerate(grads):
        np.testing.assert_allclose(g.numpy(), z[f"g{i}"], rtol=1e-5, atol=1e-5)


def _model_inputs(z, tag):
    n = int(z[f"{tag}_n"])
    idx = z[f"{tag}_op_idx"]
    r, c, v = og.coalesce(idx[0], idx[1], z[f"{tag}_op_val"], n, n)
    P = ops.csr_tensor(*og.csr_of(r, c, v, n), n, n)
    PT = ops.csr_tensor(*og.csr_transpose(r, c, v, n), n, n)
    gat_graph = og.gat_graph(z[f"{tag}_edge"], n)
    return n, P, PT, gat_graph


def test_oracle_model_matches_reference_model(golden):
    z = golden("model_cases.npz")
    for case in z["cases"]:
        tag, gname, hops = str(case).split("|")
        hops = [int(h) for h in hops.split(",")]
        n, P, PT, gat_graph = _model_inputs(z, tag)
        m = OracleCIGN(8, 24, 3, 2, hops, 0.0, 2, 0.0)
        state = {k[len(tag) + 3:]: torch.from_numpy(z[k]) for k in z.keys()
                 if k.startswith(f"{tag}_p_")}
        m.load_state_dict(state, strict=True)
        y = m(torch.from_numpy(z[f"{tag}_x"]), P, PT, gat_graph)
        np.testing.assert_allclose(y.detach().numpy(), z[f"{tag}_y"], rtol=2e-4, atol=2e-5,
                                   err_msg=str(case))
        (y * torch.from_numpy(z[f"{tag}_go"])).sum().backward()
        for name, p in m.named_parameters():
            key = f"{tag}_gp_{name}"
            if key in z:
                np.testing.assert_allclose(p.grad.numpy(), z[key], rtol=5e-4, atol=5e-5,
                                           err_msg=f"{case} {name}")


def test_gat_oracle_matches_independent_gatconv():
    g = torch.Generator().manual_seed(3)
    n, H, C = 37, 3, 8
    src = torch.randint(0, n, (150,), generator=g)
    dst = torch.randint(0, n, (150,), generator=g)
    keep = src != dst
    loops = torch.arange(n)
    edge = torch.stack([torch.cat([src[keep], loops]), torch.cat([dst[keep], loops])]).numpy()
    x = torch.randn(n, H, C, generator=g)
    att_src = torch.randn(1, H, C, generator=g) * 0.3
    att_dst = torch.randn(1, H, C, generator=g) * 0.3
    bias = torch.randn(C, generator=g) * 0.1
    (rowptr, col), _, _ = og.gat_graph(edge, n)
    a_src, a_dst = ops.attention_logits(x, att_src, att_dst)
    out, pre, m, s = ops.gat_collapsed(a_dst, a_src, rowptr, col, x, bias, 0.2, 0.0, 0)
    ref = ops.gatconv_mean_bias_silu(x, att_src, att_dst, edge, bias, 0.2)
    torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-6)


def test_gat_oracle_empty_rows_and_dropout_scaling():
    n, H, C = 5, 2, 4
    edge = np.array([[1, 2, 3], [0, 0, 1]])  # rows 2,3,4 have no in-edges
    (rowptr, col), _, _ = og.gat_graph(edge, n)
    x = torch.randn(n, H, C)
    bias = torch.randn(C)
    a = torch.randn(n, H)
    out, pre, m, s = ops.gat_collapsed(a, a, rowptr, col, x, bias, 0.2, 0.0, 0)
    torch.testing.assert_close(out[2:], torch.nn.functional.silu(bias).expand(3, C))
    assert torch.all(m[2:] == -1.0e38) and torch.all(s[2:] == 0)
