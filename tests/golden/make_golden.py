"""Generate the golden fixtures of tests/golden/ by running the REFERENCE's own
Python code (rabbit-art/CIGN) on the CPU.

    python tests/golden/make_golden.py --reference <path to the reference tree>

Only this script reads the reference tree; the fixtures it writes are small
.npz files that travel with the repository (the reference does not).  The
reference's CUDA extensions are never built or run: every call below is a
CPU-runnable path of the reference:

  * model.prepare_fixed_csr_operator + FixedCSRSpMMFunction (model.py:106-199)
    on the random operator of validate_fixedcsr.py;
  * multihop_csr_pipeline.GenericMultiHopCSRFunction (multihop_csr_pipeline.py
    :233-306) on the circulant operator of validate_a3v5.py:11-19;
  * the pack oracles legacy_pack (validate_a3.py:8-19), reference() of
    validate_cign_switch_pack.py:17-50 and validate_cign_acceleration.py:10-18;
  * legacy_block_ops (validate_a3v8.py:27-31) with p = 0;
  * generic_engine/model_cign.GraphCliffordNet with every use_fused_* False
    on the ring graph of validate_cign_acceleration.py:44-58 and on a small
    random graph with self loops.

torch_geometric is not installed, so `torch_geometric.nn` is replaced by a
stub module whose GATConv restates PyG's GATConv(concat=False) semantics
(lin without bias, att_src/att_dst [1,H,C], LeakyReLU 0.2, per-target
softmax, head mean, bias).  That GATConv is therefore not pinned by this
script; the rest of the model wiring is the reference's own code.
"""
from __future__ import annotations

import argparse
import math
import sys
import types
from pathlib import Path

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

OUT_DIR = Path(__file__).resolve().parent


# ----------------------------------------------------------- PyG stub
class _StubGATConv(nn.Module):
    def __init__(self, in_channels, out_channels, heads=1, concat=True, negative_slope=0.2,
                 dropout=0.0, add_self_loops=True, bias=True, **kwargs):
        super().__init__()
        self.in_channels, self.out_channels, self.heads = in_channels, out_channels, heads
        self.concat, self.negative_slope, self.dropout = concat, negative_slope, dropout
        self.add_self_loops = add_self_loops
        self.lin = nn.Linear(in_channels, heads * out_channels, bias=False)
        self.att_src = nn.Parameter(torch.empty(1, heads, out_channels))
        self.att_dst = nn.Parameter(torch.empty(1, heads, out_channels))
        self.bias = nn.Parameter(torch.zeros(heads * out_channels if concat else out_channels)) \
            if bias else None
        for t in (self.lin.weight, self.att_src, self.att_dst):
            a = math.sqrt(6.0 / (t.size(-2) + t.size(-1)))
            nn.init.uniform_(t, -a, a)

    def forward(self, x, edge_index):
        H, C = self.heads, self.out_channels
        xl = self.lin(x).view(-1, H, C)
        a_src = (xl * self.att_src).sum(-1)
        a_dst = (xl * self.att_dst).sum(-1)
        src, dst = edge_index[0], edge_index[1]
        n = x.size(0)
        logit = F.leaky_relu(a_src[src] + a_dst[dst], self.negative_slope)
        m = torch.full((n, H), -float("inf")).scatter_reduce(
            0, dst[:, None].expand(-1, H), logit.detach(), reduce="amax", include_self=True)
        ex = torch.exp(logit - m[dst])
        s = torch.zeros((n, H)).index_add(0, dst, ex)
        alpha = ex / s[dst]
        alpha = F.dropout(alpha, p=self.dropout, training=self.training)
        out = torch.zeros((n, H, C)).index_add(0, dst, alpha[:, :, None] * xl[src])
        out = out.reshape(n, H * C) if self.concat else out.mean(1)
        return out + self.bias if self.bias is not None else out


def install_pyg_stub():
    tg = types.ModuleType("torch_geometric")
    tgnn = types.ModuleType("torch_geometric.nn")
    tgnn.GATConv = _StubGATConv
    tgnn.FusedGATConv = _StubGATConv
    tg.nn = tgnn
    sys.modules["torch_geometric"] = tg
    sys.modules["torch_geometric.nn"] = tgnn


def t2n(t):
    return t.detach().cpu().numpy()


# ----------------------------------------------------------- fixtures
def fixed_csr(ref_model):
    torch.manual_seed(42)
    n, e, f = 300, 2400, 16
    row = torch.randint(0, n, (e,))
    col = torch.randint(0, n, (e,))
    val = torch.rand(e)
    coo = torch.sparse_coo_tensor(torch.stack([row, col]), val, (n, n))
    op = ref_model.prepare_fixed_csr_operator(coo)
    x = torch.randn(n, f, requires_grad=True)
    y = ref_model.FixedCSRSpMMFunction.apply(x, op.csr, op.csr_t)
    gy = torch.randn_like(y)
    (y * gy).sum().backward()
    np.savez_compressed(
        OUT_DIR / "fixedcsr_random.npz",
        coo_row=t2n(row), coo_col=t2n(col), coo_val=t2n(val), n=n,
        crow=t2n(op.csr.crow_indices()), col=t2n(op.csr.col_indices()), val=t2n(op.csr.values()),
        crow_t=t2n(op.csr_t.crow_indices()), col_t=t2n(op.csr_t.col_indices()),
        val_t=t2n(op.csr_t.values()), x=t2n(x), y=t2n(y), gy=t2n(gy), gx=t2n(x.grad))


def multihop(ref_model, ref_mh):
    n, d = 320, 12
    offsets = torch.tensor([0, 1, -1, 7, -7, 31, -31, 127, -127])
    row = torch.arange(n).repeat_interleave(offsets.numel())
    col = ((torch.arange(n)[:, None] + offsets[None, :]) % n).reshape(-1)
    val = torch.full((row.numel(),), 1.0 / offsets.numel())
    coo = torch.sparse_coo_tensor(torch.stack([row, col]), val, (n, n)).coalesce()
    base = ref_model.prepare_fixed_csr_operator(coo)
    out = {"coo_row": t2n(row), "coo_col": t2n(col), "coo_val": t2n(val), "n": n}
    torch.manual_seed(42)
    for name, powers in (("p123", (1, 2, 3)), ("p1248", (1, 2, 4, 8)), ("p0_2_5", (0, 2, 5))):
        op = ref_mh.GenericMultiHopCSRGraphOperator(base, dense_cols=d, powers=powers)
        x = torch.randn(n, d, requires_grad=True)
        res = ref_mh.generic_multihop_csr(op, x)
        loss = 0.0
        for p in op.positive_powers:
            g = torch.randn(n, d)
            out[f"{name}_g{p}"] = t2n(g)
            out[f"{name}_y{p}"] = t2n(res[p])
            loss = loss + (res[p] * g).sum()
        loss.backward()
        out[f"{name}_x"] = t2n(x)
        out[f"{name}_gx"] = t2n(x.grad)
    np.savez_compressed(OUT_DIR / "multihop_circulant.npz", **out)


def packs(val_a3, val_switch, val_accel):
    out = {}
    cases = []
    # CIGN ("new" interaction, no outer): validate_cign_acceleration.py:38-44
    for k, d in [(1, 24), (2, 32), (3, 24), (3, 64), (5, 24)]:
        for w in ("old", "new"):
            cases.append(("cign", k, d, w, lambda h, c, p, a, w=w: val_accel.reference(h, c, p, a, w)))
    # tanh switch, both interactions: validate_cign_switch_pack.py:17-50
    for inter in ("old", "new"):
        for w in ("old", "new"):
            cases.append((f"switch_{inter}", 3, 64, w,
                          lambda h, c, p, a, i=inter, w=w: val_switch.reference(h, c, p, a, i, w)))
    # old interaction pack: validate_a3.py:8-19
    cases.append(("legacy", 3, 32, "old", lambda h, c, p, a: val_a3.legacy_pack(h, c, p, a)))
    cases.append(("legacy", 4, 16, "old", lambda h, c, p, a: val_a3.legacy_pack(h, c, p, a)))
    names = []
    for i, (kind, k, d, w, fn) in enumerate(cases):
        torch.manual_seed(1000 + i)
        n = 17 + i
        raw = [torch.randn(n, d), torch.randn(n, d)] + [torch.randn(n, 2 * d) for _ in range(k)] + \
            [torch.randn(n, k)]
        leaves = [r.clone().requires_grad_(True) for r in raw]
        alpha = torch.softmax(leaves[-1], -1)
        y = fn(leaves[0], leaves[1], leaves[2:-1], alpha)
        go = torch.randn_like(y)
        grads = torch.autograd.grad(y, leaves, go)
        tag = f"c{i}"
        names.append(f"{tag}|{kind}|{k}|{d}|{w}")
        for j, r in enumerate(raw):
            out[f"{tag}_in{j}"] = t2n(r)
        out[f"{tag}_y"] = t2n(y)
        out[f"{tag}_go"] = t2n(go)
        for j, g in enumerate(grads):
            out[f"{tag}_g{j}"] = t2n(g)
    out["cases"] = np.array(names)
    np.savez_compressed(OUT_DIR / "pack_cases.npz", **out)


def block_ops(val_a3v8):
    torch.manual_seed(1234)
    n, d = 64, 48
    raw = [torch.randn(n, d), torch.randn(n, d), torch.randn(n, d)]
    params = [1.0 + 0.1 * torch.randn(d), 0.1 * torch.randn(d), 1.0 + 0.1 * torch.randn(d),
              0.1 * torch.randn(d), 0.49 + 0.05 * torch.randn(d)]
    leaves = [t.clone().requires_grad_(True) for t in raw + params]
    H, Cg, G, hw, hb, cw, cb, gamma = leaves
    Hn, Cn, Y = val_a3v8.legacy_block_ops(H, Cg, G, hw, hb, cw, cb, gamma, 0.0, 1e-5)
    gos = [torch.randn_like(t) for t in (Hn, Cn, Y)]
    loss = sum((a * b).sum() for a, b in zip((Hn, Cn, Y), gos))
    grads = torch.autograd.grad(loss, leaves)
    out = {f"in{i}": t2n(t) for i, t in enumerate(raw + params)}
    out.update({"Hn": t2n(Hn), "Cn": t2n(Cn), "Y": t2n(Y)})
    out.update({f"go{i}": t2n(t) for i, t in enumerate(gos)})
    out.update({f"g{i}": t2n(t) for i, t in enumerate(grads)})
    np.savez_compressed(OUT_DIR / "block_ops.npz", **out)


def models(model_cign):
    out = {}
    names = []
    graphs = {}
    n = 23
    graphs["ring"] = (n, torch.stack([torch.arange(n), torch.arange(n).roll(1)]))
    g = torch.Generator().manual_seed(5)
    m = 40
    e = torch.randint(0, m, (2, 160), generator=g)
    e = e[:, e[0] != e[1]]
    loops = torch.arange(m)
    graphs["er40"] = (m, torch.cat([e, torch.stack([loops, loops])], dim=1))
    for gname, hops in (("ring", [1, 2, 3]), ("ring", [1, 2, 4, 8, 16]), ("er40", [1, 2, 3]),
                        ("er40", [1, 3])):
        nn_, edge = graphs[gname]
        # symmetric normalised operator so that powers stay bounded
        ones = torch.ones(edge.size(1))
        A = torch.sparse_coo_tensor(edge, ones, (nn_, nn_)).coalesce()
        A = (A + A.t()).coalesce()
        deg = torch.sparse.sum(A, 1).to_dense().clamp(min=1)
        idx = A.indices()
        vals = A.values() / torch.sqrt(deg[idx[0]] * deg[idx[1]])
        operator = torch.sparse_coo_tensor(idx, vals, (nn_, nn_)).coalesce()
        torch.manual_seed(42)
        x = torch.randn(nn_, 8)
        kwargs = dict(in_dim=8, hidden_dim=24, out_dim=3, num_layers=2, dropout=0.0, gat_dropout=0.0,
                      gat_heads=2, hop_scales=hops)
        model = model_cign.build_model(**kwargs, use_fused_clifford_pack=False)
        with torch.no_grad():
            for blk in model.blocks:
                blk.context_gat.bias.normal_(0, 0.1)
        y = model(x, edge, operator)
        go = torch.randn_like(y)
        (y * go).sum().backward()
        tag = f"m{len(names)}"
        names.append(f"{tag}|{gname}|{','.join(map(str, hops))}")
        out[f"{tag}_x"] = t2n(x)
        out[f"{tag}_edge"] = t2n(edge)
        out[f"{tag}_op_idx"] = t2n(operator.indices())
        out[f"{tag}_op_val"] = t2n(operator.values())
        out[f"{tag}_n"] = nn_
        out[f"{tag}_y"] = t2n(y)
        out[f"{tag}_go"] = t2n(go)
        for pname, p in model.named_parameters():
            out[f"{tag}_p_{pname}"] = t2n(p)
            if p.grad is not None:
                out[f"{tag}_gp_{pname}"] = t2n(p.grad)
    out["cases"] = np.array(names)
    np.savez_compressed(OUT_DIR / "model_cases.npz", **out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference source tree")
    args = ap.parse_args()
    ref = Path(args.reference).resolve()
    sys.dont_write_bytecode = True
    install_pyg_stub()
    import os
    os.environ.update(CIGN_ALPHA_SCORE_MODE="new", CIGN_INTERACTION_MODE="new",
                      CIGN_ALPHA_WEIGHTING_MODE="old", CIGN_OUTER_NONLINEARITY="none")
    sys.path.insert(0, str(ref))
    import model as ref_model  # noqa: E402  (reference model.py)
    import multihop_csr_pipeline as ref_mh  # noqa: E402
    import validate_a3  # noqa: E402
    import validate_a3v8  # noqa: E402
    import validate_cign_switch_pack  # noqa: E402
    fixed_csr(ref_model)
    multihop(ref_model, ref_mh)
    block_ops(validate_a3v8)
    # validate_cign_acceleration and model_cign live next to generic_engine/
    sys.path.insert(0, str(ref / "generic_engine"))
    for mod in ("model", "multihop_csr_pipeline", "fused_clifford_pack", "fused_gat_sideops",
                "fused_block_ops", "collapsed_gat", "chunked_dgnn_gat"):
        sys.modules.pop(mod, None)
    import validate_cign_acceleration  # noqa: E402
    packs(validate_a3, validate_cign_switch_pack, validate_cign_acceleration)
    import model_cign  # noqa: E402
    models(model_cign)
    for p in sorted(OUT_DIR.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
