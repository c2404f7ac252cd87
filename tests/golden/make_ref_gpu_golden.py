"""Golden fixtures and an A/B timing table from the REFERENCE's own CUDA
kernels, run on a B200 -- TEST INFRASTRUCTURE.

    python tests/golden/make_ref_gpu_golden.py --out <dir>          # fixtures
    python tests/golden/make_ref_gpu_golden.py --ab <file.json>     # A/B timings

Needs a GPU and the reference's extensions in oracle/_ref/ (built from the
reference's unchanged sources by oracle/build_ref.py; they travel with the
working tree, the reference tree does not).  The reference kernels are called
through their own pybind entry points with the argument order of their Python
wrappers.

Fixtures (small seeded cases; every array the reference returns is stored):

  ref_gat_family.npz  collapsed GAT (collapsed_gat_ext, the only shape it
      accepts: H=6, C=256, collapsed_gat.cpp:67-68) on a 128-node graph with
      a 100-edge hub row and a 70-edge hub column, attn_drop 0 and 0.5:
      out, pre, edge_max, edge_sum, the uint8 [nnz,H] keep mask and the four
      gradients; attention logits and head-mean + bias + SiLU
      (fused_gat_sideops_ext) forward and backward on the same [N,6,256].
  ref_block_ops_gpu.npz  dropout-LN, add-LN and dropout-gamma-residual,
      forward and backward with p = 0.5, at D=256 (fused_block_ops_ext, the
      D=256 kernels) and D=96 (the 1<=D<=256 kernels inlined in
      fused_block_ops.py:14-15), uint8 masks included.

A/B (--ab): the reference kernel and this repository's kernel for the same op
on the cfg2 graph (N=24,492, power-law) at the shapes the reference accepts,
CUDA-event times (median of 20 after 3 warm-ups, L2 flushed before every
call), written as JSON.
"""
from __future__ import annotations

import argparse
import json
import statistics
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

from oracle.build_ref import load_extension  # noqa: E402

GAT_SEED = 0x1234_5678_9ABC_DEF
LN_SEED = 0x0DDB_A11_5EED
GAMMA_SEED = 0x5EED_0F_6A33A


def n2(t):
    return t.detach().cpu().numpy()


def gat_graph(n: int):
    """Power-law edges plus a hub destination (row 0 receives 100 edges) and
    a hub source (node 1 feeds 70 rows); PyG GAT self-loop handling; CSR by
    destination, CSC and perm from this repository's to_graph_format (the
    CSR/CSC/perm convention of model_cign.py:1116-1142)."""
    from cign_b200 import synth
    from cign_b200.graph_operator import prepare_gat_edge_index, to_graph_format
    edge = synth.powerlaw_graph(n, 600, seed=11)
    g = torch.Generator().manual_seed(5)
    hub_in = torch.stack([torch.randperm(n, generator=g)[:100], torch.zeros(100, dtype=torch.long)])
    hub_out = torch.stack([torch.ones(70, dtype=torch.long), torch.randperm(n, generator=g)[:70]])
    ei = prepare_gat_edge_index(torch.cat([edge, hub_in, hub_out], 1), n)
    (rp, c), (r, cp), perm = to_graph_format(ei.flip(0), n)
    return [t.to(torch.int32).contiguous() for t in (rp, c, cp, r, perm)]


def make_gat_family(dev) -> dict:
    ext = load_extension("ref_collapsed_gat")
    side = load_extension("ref_gat_sideops")
    n, H, C = 128, 6, 256
    rp, c, cp, r, perm = gat_graph(n)
    g = torch.Generator().manual_seed(2024)
    x = torch.randn(n, H, C, generator=g)
    a_row = torch.randn(n, H, generator=g)
    a_col = torch.randn(n, H, generator=g)
    bias = torch.randn(C, generator=g) * 0.1
    gy = torch.randn(n, C, generator=g)
    att_src = torch.randn(1, H, C, generator=g) * 0.1
    att_dst = torch.randn(1, H, C, generator=g) * 0.1
    g_src = torch.randn(n, H, generator=g)
    g_dst = torch.randn(n, H, generator=g)
    slope = 0.2
    out = dict(rowptr=n2(rp), col=n2(c), colptr=n2(cp), row=n2(r), perm=n2(perm), n=n, H=H, C=C,
               negative_slope=slope, attn_row=n2(a_row), attn_col=n2(a_col), in_feat=n2(x),
               bias=n2(bias), grad_y=n2(gy), att_src=n2(att_src), att_dst=n2(att_dst),
               grad_src=n2(g_src), grad_dst=n2(g_dst), seed_p50=np.uint64(GAT_SEED))
    d = {k: v.to(dev) for k, v in dict(rp=rp, c=c, cp=cp, r=r, perm=perm, x=x, a_row=a_row,
                                         a_col=a_col, bias=bias, gy=gy, att_src=att_src,
                                         att_dst=att_dst, g_src=g_src, g_dst=g_dst).items()}
    for tag, p, seed in (("p0", 0.0, 0), ("p50", 0.5, GAT_SEED)):
        y, pre, emax, esum, mask = ext.forward(d["a_row"], d["a_col"], d["rp"], d["c"], slope,
                                               d["x"], d["bias"], p, seed)
        gfeat, grow, gcol, gbias = ext.backward(slope, p, d["rp"], d["c"], d["cp"], d["r"],
                                                d["perm"], emax, esum, mask, d["x"], d["a_row"],
                                                d["a_col"], pre, d["gy"])
        for k, v in dict(out=y, pre=pre, edge_max=emax, edge_sum=esum, edge_mask=mask,
                         grad_feat=gfeat, grad_attn_row=grow, grad_attn_col=gcol,
                         grad_bias=gbias).items():
            out[f"{k}_{tag}"] = n2(v)
    a_s, a_d = side.attention_forward(d["x"], d["att_src"], d["att_dst"])
    gx, gas, gad = side.attention_backward(d["g_src"], d["g_dst"], d["x"], d["att_src"],
                                           d["att_dst"])
    hy, hpre = side.head_silu_forward(d["x"], d["bias"])
    hgo, hgb = side.head_silu_backward(d["gy"], hpre, H)
    out.update(alpha_src=n2(a_s), alpha_dst=n2(a_d), logits_grad_x=n2(gx),
               logits_grad_att_src=n2(gas), logits_grad_att_dst=n2(gad), head_y=n2(hy),
               head_pre=n2(hpre), head_grad_out=n2(hgo), head_grad_bias=n2(hgb))
    torch.cuda.synchronize()
    return out


def make_block_ops(dev) -> dict:
    out = {}
    for D, name in ((256, "ref_block_ops_d256"), (96, "ref_block_ops_general")):
        ext = load_extension(name)
        n, p, eps = 128, 0.5, 1e-5
        g = torch.Generator().manual_seed(77 + D)
        t = {k: torch.randn(n, D, generator=g) for k in ("x", "a", "b", "h", "gm", "gy")}
        t.update(w=1.0 + 0.1 * torch.randn(D, generator=g), bb=0.1 * torch.randn(D, generator=g),
                 gamma=0.1 * torch.randn(D, generator=g))
        d = {k: v.to(dev) for k, v in t.items()}
        pre = f"d{D}_"
        for k, v in t.items():
            out[pre + k] = n2(v)
        y, mean, rstd, mask = ext.dropout_layernorm_forward(d["x"], d["w"], d["bb"], p, eps,
                                                            LN_SEED)
        dx, gw, gb = ext.dropout_layernorm_backward(d["gy"], d["x"], d["w"], mean, rstd, mask, p)
        out.update({pre + "dln_y": n2(y), pre + "dln_mean": n2(mean), pre + "dln_rstd": n2(rstd),
                    pre + "dln_mask": n2(mask), pre + "dln_dx": n2(dx), pre + "dln_gw": n2(gw),
                    pre + "dln_gb": n2(gb)})
        y, mean, rstd = ext.add_layernorm_forward(d["a"], d["b"], d["w"], d["bb"], eps)
        dz, gw, gb = ext.add_layernorm_backward(d["gy"], d["a"], d["b"], d["w"], mean, rstd)
        out.update({pre + "aln_y": n2(y), pre + "aln_mean": n2(mean), pre + "aln_rstd": n2(rstd),
                    pre + "aln_dz": n2(dz), pre + "aln_gw": n2(gw), pre + "aln_gb": n2(gb)})
        y, mask = ext.dropout_gamma_residual_forward(d["h"], d["gm"], d["gamma"], p, GAMMA_SEED)
        gg, ggamma = ext.dropout_gamma_residual_backward(d["gy"], d["gm"], d["gamma"], mask, p)
        out.update({pre + "gres_y": n2(y), pre + "gres_mask": n2(mask), pre + "gres_gg": n2(gg),
                    pre + "gres_ggamma": n2(ggamma)})
    out.update(p=0.5, eps=1e-5, ln_seed=np.uint64(LN_SEED), gamma_seed=np.uint64(GAMMA_SEED))
    torch.cuda.synchronize()
    return out


# ----------------------------------------------------------------------- A/B
class Timer:
    def __init__(self, dev, reps=20, warmup=3):
        self.reps, self.warmup = reps, warmup
        self.flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)

    def __call__(self, fn) -> float:
        for _ in range(self.warmup):
            fn()
        times = []
        for _ in range(self.reps):
            self.flush.fill_(1.0)
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            b.synchronize()
            times.append(a.elapsed_time(b))
        return statistics.median(times)


def ab_table(dev) -> dict:
    from cign_b200 import _pack, collapsed_gat, fused_block_ops, fused_gat_sideops, synth
    from cign_b200.graph_operator import (build_sparse_normalized_adjacency,
                                          prepare_fixed_csr_operator, prepare_gat_edge_index,
                                          to_graph_format)
    from cign_b200.multihop_csr_pipeline import _csr_parts_int32, _NativePlan
    from cign_b200.plans import gat_plan_for

    cfg = synth.CONFIGS["cfg2"]
    n = cfg.num_nodes
    edge = synth.make_edges(cfg).to(dev)
    ei, adj = build_sparse_normalized_adjacency(edge, n)
    base = prepare_fixed_csr_operator(adj)
    gat_e = prepare_gat_edge_index(ei, n)
    (rp, c), (r, cp), perm = to_graph_format(gat_e.flip(0), n)
    rp, c, r, cp, perm = (t.to(torch.int32).contiguous() for t in (rp, c, r, cp, perm))
    timer = Timer(dev)
    rows = []

    def row(op, shape, ref_fn, ours_fn, note=""):
        ref_ms, ours_ms = timer(ref_fn), timer(ours_fn)
        rows.append(dict(op=op, shape=shape, reference_ms=round(ref_ms, 4),
                         ours_ms=round(ours_ms, 4), speedup=round(ref_ms / ours_ms, 2), note=note))
        print(json.dumps(rows[-1]), flush=True)

    g = torch.Generator(device=dev).manual_seed(0)

    def rnd(*shape):
        return torch.randn(*shape, generator=g, device=dev)

    # multihop SpMM: cuSPARSE ALG2 plan (multihop_csr_pipeline_cuda.cu:113-322) vs ours
    mh = load_extension("ref_multihop_csr")
    p = _csr_parts_int32(base.csr)
    pt = _csr_parts_int32(base.csr_t)
    for F in (1024, 512, 128):
        ref_plan = mh.MultiHopCsrPlan(p[0], p[1], p[2], pt[0], pt[1], pt[2], n, F, 2)
        ref_plan.prepare(torch.empty(n, F, device=dev))
        ours = _NativePlan(p, pt, n, F, 2)
        x = rnd(n, F)
        gs = [rnd(n, F) for _ in range(3)]
        row("multihop fwd (3 hops)", f"N={n} F={F}", lambda: ref_plan.forward3(x),
            lambda: ours.forward3(x))
        row("multihop bwd (3 hops)", f"N={n} F={F}", lambda: ref_plan.backward3(*gs),
            lambda: ours.backward3(*gs))

    # collapsed GAT at the reference's only shape (H=6, C=256), p = 0.5
    cg = load_extension("ref_collapsed_gat")
    H, C = 6, 256
    x = rnd(n, H, C)
    a_row, a_col = rnd(n, H), rnd(n, H)
    bias = rnd(C) * 0.1
    gy = rnd(n, C)
    plan = gat_plan_for(rp, c, r, cp, perm)
    st = {}

    def ref_fwd():
        st["ref"] = cg.forward(a_row, a_col, rp, c, 0.2, x, bias, 0.5, GAT_SEED)

    def ours_fwd():
        st["ours"] = collapsed_gat.gat_forward_raw(plan, a_row, a_col, x, bias, 0.2, 0.5, GAT_SEED)

    row("collapsed GAT fwd", f"N={n} nnz={int(c.numel())} H=6 C=256 p=0.5", ref_fwd, ours_fwd)
    y, pre, emax, esum, mask = st["ref"]
    _, opre, oemax, oesum = st["ours"]
    row("collapsed GAT bwd", f"N={n} nnz={int(c.numel())} H=6 C=256 p=0.5",
        lambda: cg.backward(0.2, 0.5, rp, c, cp, r, perm, emax, esum, mask, x, a_row, a_col, pre,
                            gy),
        lambda: collapsed_gat.gat_backward_raw(plan, a_row, a_col, x, opre, oemax, oesum, gy, 0.2,
                                               0.5, GAT_SEED))

    side = load_extension("ref_gat_sideops")
    att_s, att_d = rnd(1, H, C) * 0.1, rnd(1, H, C) * 0.1
    g_s, g_d = rnd(n, H), rnd(n, H)
    row("attention logits fwd", f"N={n} H=6 C=256", lambda: side.attention_forward(x, att_s, att_d),
        lambda: fused_gat_sideops.attention_logits_forward(x, att_s, att_d))
    row("attention logits bwd", f"N={n} H=6 C=256",
        lambda: side.attention_backward(g_s, g_d, x, att_s, att_d),
        lambda: fused_gat_sideops.attention_logits_backward(g_s, g_d, x, att_s, att_d))

    # block ops at D=256 (the reference's specialised kernels)
    blk = load_extension("ref_block_ops_d256")
    D = 256
    xb, ab, bb, gyb = rnd(n, D), rnd(n, D), rnd(n, D), rnd(n, D)
    w, b0, gamma = 1.0 + 0.1 * rnd(D), 0.1 * rnd(D), 0.1 * rnd(D)
    ry, rmean, rrstd, rmask = blk.dropout_layernorm_forward(xb, w, b0, 0.5, 1e-5, LN_SEED)
    _, omean, orstd = fused_block_ops.dropout_ln_forward(xb, w, b0, 0.5, 1e-5, LN_SEED)
    row("dropout-LN fwd", f"N={n} D=256 p=0.5",
        lambda: blk.dropout_layernorm_forward(xb, w, b0, 0.5, 1e-5, LN_SEED),
        lambda: fused_block_ops.dropout_ln_forward(xb, w, b0, 0.5, 1e-5, LN_SEED))
    row("dropout-LN bwd", f"N={n} D=256 p=0.5",
        lambda: blk.dropout_layernorm_backward(gyb, xb, w, rmean, rrstd, rmask, 0.5),
        lambda: fused_block_ops.dropout_ln_backward(gyb, xb, w, omean, orstd, 0.5, LN_SEED))
    _, amean, arstd = blk.add_layernorm_forward(ab, bb, w, b0, 1e-5)
    row("add-LN fwd", f"N={n} D=256", lambda: blk.add_layernorm_forward(ab, bb, w, b0, 1e-5),
        lambda: fused_block_ops.add_ln_forward(ab, bb, w, b0, 1e-5))
    row("add-LN bwd", f"N={n} D=256",
        lambda: blk.add_layernorm_backward(gyb, ab, bb, w, amean, arstd),
        lambda: fused_block_ops.add_ln_backward(gyb, ab, bb, w, amean, arstd))
    _, gmask = blk.dropout_gamma_residual_forward(xb, ab, gamma, 0.5, GAMMA_SEED)
    row("dropout-gamma-residual fwd", f"N={n} D=256 p=0.5",
        lambda: blk.dropout_gamma_residual_forward(xb, ab, gamma, 0.5, GAMMA_SEED),
        lambda: fused_block_ops.gamma_residual_forward(xb, ab, gamma, 0.5, GAMMA_SEED))
    row("dropout-gamma-residual bwd", f"N={n} D=256 p=0.5",
        lambda: blk.dropout_gamma_residual_backward(gyb, ab, gamma, gmask, 0.5),
        lambda: fused_block_ops.gamma_residual_backward(gyb, ab, gamma, 0.5, GAMMA_SEED))

    # CIGN pack, K=3 (interaction new, weighting old: the production mode), D=512
    pk = load_extension("ref_cign_pack3")
    D = 512
    Hn, Cn = rnd(n, D), rnd(n, D)
    props = [rnd(n, 2 * D) for _ in range(3)]
    alpha = torch.softmax(rnd(n, 3), 1).contiguous()
    gout = rnd(n, 6 * D)
    row("CIGN pack fwd (K=3, new/old)", f"N={n} D=512",
        lambda: pk.forward(Hn, Cn, *props, alpha, 1, 0),
        lambda: _pack.pack_forward(Hn, Cn, props, alpha, 1, 0, 0))
    row("CIGN pack bwd (K=3, new/old)", f"N={n} D=512",
        lambda: pk.backward(gout, Hn, Cn, *props, alpha, 1, 0),
        lambda: _pack.pack_backward(gout, Hn, Cn, props, alpha, 1, 0, 0, True))
    pkk = load_extension("ref_cign_pack_k")
    Pst = torch.stack(props, 1).contiguous()
    row("CIGN generic-K pack fwd (K=3)", f"N={n} D=512",
        lambda: pkk.forward(Hn, Cn, Pst, alpha),
        lambda: _pack.pack_forward(Hn, Cn, props, alpha, 1, 0, 0),
        note="reference output layout [N,2D] (new weighting); ours timed in the K=3 old-weighting layout")
    return dict(graph=dict(workload=cfg.name, nodes=n, nnz_P=int(base.nnz), nnz_gat=int(c.numel())),
                device=torch.cuda.get_device_name(dev), rows=rows,
                timing="CUDA events, median of 20 after 3 warm-ups, 256 MiB L2 flush before each call")


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=None, help="directory for the .npz fixtures")
    ap.add_argument("--ab", default=None, help="JSON file for the A/B timing table")
    args = ap.parse_args(argv)
    if not torch.cuda.is_available():
        raise SystemExit("needs a CUDA GPU")
    dev = torch.device("cuda", 0)
    torch.backends.cuda.matmul.allow_tf32 = False
    if args.out:
        out = Path(args.out)
        out.mkdir(parents=True, exist_ok=True)
        np.savez_compressed(out / "ref_gat_family.npz", **make_gat_family(dev))
        np.savez_compressed(out / "ref_block_ops_gpu.npz", **make_block_ops(dev))
        print(f"fixtures written to {out}")
    if args.ab:
        res = ab_table(dev)
        Path(args.ab).parent.mkdir(parents=True, exist_ok=True)
        Path(args.ab).write_text(json.dumps(res, indent=1))
        print(f"A/B table written to {args.ab}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
