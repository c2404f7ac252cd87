"""CIGN training-step benchmark on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload ("cfg2", the headline configuration): full CIGN forward + backward +
Adam step, fp32 (TF32 dense GEMMs as the reference's default), on a seeded
synthetic power-law graph (N=24,492, 186,100 directed edges, exponent 2.5),
features [N,300] ~ N(0,1), 5 uniform classes, hidden 512 (= 64 channels x 8
blades), hops {1,2,3}, 4 heads, 2 layers, dropout 0.5 (GAT dropout 0.5),
50/25/25 split.  Random-init weights; synthetic data stands in for the
reference's dataset.

Metric: GTEPS = SpMM edge-passes per step (L*K forward + L*K transposed
backward passes over nnz(P)) / step time / 1e9; the epoch time in ms is
ms_per_step.  `value` is device-timed with inputs resident in HBM; `e2e`
is the same step through the public API with the features copied from
pinned host memory and the loss read back every step.

--impl reference times the reference's own CPU path (its torch ops restated
in oracle/, run on all host cores) on the same workload graph, whole, for up
to --steps steps within --cpu-budget-s seconds; there is no GPU in that arm.
The cpu_baseline object of the GPU arm is the same runner for 3 steps.

roofline.epoch_frac = T_roof / ms_per_step, T_roof = sum over every kernel of
the step (step_roofline_items) of max(compulsory bytes / HBM peak, FLOPs /
TF32 peak).

With --gpus N > 1 (torchrun, NCCL) the graph is row-partitioned over the
ranks with a halo exchange per hop and per GAT layer and one gradient
all-reduce per step: cfg2 scales weakly (an N x cfg2 graph, a cfg2-sized row
range per rank), other workloads (--workload cfg4, the 2.45M-node RMAT
graph) strongly.  `value` is the whole job's edge-passes over the slowest
rank's time.  Workloads above GRAPH_CAPTURE_MAX_NODES nodes run eagerly;
smaller ones replay each step as one CUDA graph (--eager to opt out).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch
import torch.nn.functional as F

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PEAKS_PATH = ROOT / "MEASURED_PEAKS.json"
TRAFFIC_PATH = ROOT / "profiles" / "traffic.json"
FALLBACK_HBM_GBS = 6650.0
L2_FLUSH_BYTES = 256 << 20
GRAPH_CAPTURE_MAX_NODES = 1_000_000  # larger workloads run eagerly


# ------------------------------------------------------------------ helpers
def load_peaks():
    if PEAKS_PATH.exists():
        try:
            d = json.loads(PEAKS_PATH.read_text())
            return float(d["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


FALLBACK_BF16_SUSTAINED_TFLOPS = 1400.0


def load_tf32_peak():
    """Dense TF32 tensor-core peak (TFLOP/s) for kernels inside a long step:
    the measured sustained cuBLAS bf16 rate halved (TF32 issues at half the
    bf16 rate on sm_100), else the fallback figure halved."""
    if PEAKS_PATH.exists():
        try:
            d = json.loads(PEAKS_PATH.read_text())
            return float(d["bf16_tflops_sustained"]) / 2.0, "measured bf16 sustained / 2"
        except Exception:
            pass
    return FALLBACK_BF16_SUSTAINED_TFLOPS / 2.0, "fallback bf16 sustained / 2"


def step_roofline_items(cfg, nnz, nnz_g):
    """Every kernel of one training step of the model as this repository runs
    it (forward, CE loss, backward, fused Adam), with its compulsory HBM bytes
    (each tensor it touches read or written once) and its FLOPs (GEMMs only;
    the other kernels have arithmetic intensity < 1 flop/byte).  Returns a
    list of (name, launches per step, bytes per launch, flops per launch)."""
    N, D, H, K, L = cfg.num_nodes, cfg.hidden_dim, cfg.heads, len(cfg.hops), cfg.layers
    I, Cls, F2 = cfg.in_dim, cfg.num_classes, 2 * cfg.hidden_dim
    S = L + 1                                         # JK states
    HD = H * D
    gemm = lambda m, n, k: (4 * (m * k + k * n + m * n), 2 * m * n * k)  # noqa: E731
    it = []

    def add(name, count, nbytes, flops=0):
        it.append((name, count, int(nbytes), int(flops)))

    # forward, net input
    add("input dropout", 1, 9 * N * I)
    add("input projections (one stacked GEMM)", 1, *gemm(N, 2 * D, I))
    add("input SiLU mix", 1, 12 * N * D)
    # forward, per block
    add("dropout-LN fwd", L, 8 * N * D + 8 * N)
    add("GAT logits (row dots of x with W_h^T att)", L, gemm(N, 2 * H, D)[0])
    add("GAT aggregate fwd", L, algorithmic_bytes("gat_agg_fwd", N, nnz, H=H, D=D, nnz_g=nnz_g))
    add("GAT z.M (GEMM)", L, *gemm(N, D, HD))
    add("GAT bias+SiLU + add-LN fwd", L, 16 * N * D + 8 * N)
    add("k-hop SpMM fwd hop", L * K, algorithmic_bytes("spmm", N, nnz, F=F2))
    add("hop gate + pack fwd", L, algorithmic_bytes("gate_pack_fwd", N, nnz, K=K, D=D))
    add("proj (GEMM)", L, *gemm(N, D, 2 * K * D))
    add("dropout-gamma-residual fwd", L, 12 * N * D)
    # forward, net output and loss
    add("JK LayerNorm fwd", 1, 8 * N * S * D + 8 * N)
    add("output dropout", 1, 9 * N * S * D)
    add("classifier (GEMM)", 1, *gemm(N, Cls, S * D))
    add("cross-entropy fwd+bwd", 1, 12 * N * Cls)
    # backward, net output
    add("classifier dgrad (GEMM)", 1, *gemm(N, S * D, Cls))
    add("classifier wgrad (GEMM)", 1, *gemm(Cls, S * D, N))
    add("output dropout bwd", 1, 9 * N * S * D)
    add("JK LayerNorm bwd (+ parameter pass)", 1, 20 * N * S * D + 8 * N)
    # backward, per block
    # block states H_0 .. H_{L-1}: the JK LayerNorm's gradient meets the next
    # block's (the block node adds its own residual share in-kernel)
    add("block-state gradient sums", L, 12 * N * D)
    add("dropout-gamma-residual bwd", L, 12 * N * D)
    add("proj dgrad (GEMM)", L, *gemm(N, 2 * K * D, D))
    add("proj wgrad (GEMM)", L, *gemm(D, 2 * K * D, N))
    add("proj bias colsum", L, 4 * N * D)
    add("pack bwd", L, algorithmic_bytes("pack_bwd", N, nnz, K=K, D=D))
    add("k-hop SpMM bwd hop (+g fused)", L * (K - 1), algorithmic_bytes("spmm_add", N, nnz, F=F2))
    add("k-hop SpMM bwd hop", L, algorithmic_bytes("spmm", N, nnz, F=F2))
    add("hop gate bwd (+ gradient adds)", L, 24 * N * D + 8 * N * K)
    add("GAT bias+SiLU + add-LN bwd (+ parameter sums, grad H_norm += in place)", L,
        24 * N * D + 8 * N)
    add("GAT grad z (GEMM)", L, *gemm(N, HD, D))
    add("GAT aggregate bwd", L, algorithmic_bytes("gat_agg_bwd", N, nnz, H=H, C=D, D=D,
                                                   nnz_g=nnz_g))
    add("GAT lin wgrad (GEMM)", L, *gemm(HD, D, N))
    g_in = gemm(N, D, HD)
    add("GAT input dgrad (GEMM, beta = 1 into grad H_norm)", L, g_in[0] + 4 * N * D, g_in[1])
    add("GAT logits bwd (row dots, added into grad x)", L, 12 * N * D + 8 * N * H)
    add("dropout-LN bwd (+ the residual's gradient)", L, 16 * N * D + 8 * N)
    # backward, net input
    add("input SiLU mix bwd", 1, 20 * N * D)
    add("input projections wgrad (one GEMM)", 1, *gemm(2 * D, I, N))
    add("input projections bias colsum", 1, 8 * N * D)
    # optimizer: fused Adam reads param, grad, exp_avg, exp_avg_sq, writes three
    params = (2 * (I * D + D) + 1 + L * (4 * D + HD * D + 2 * H * D + D + 2 * K * D * D + D
                                     + 2 * D * K + K + D) + 2 * S * D + S * D * Cls + Cls)
    add("Adam (fused)", 1, 28 * params)
    return it


def step_roofline(cfg, nnz, nnz_g, ms_per_step, hbm_gbs, tf32_tflops):
    """T_roof = sum over the step's kernels of max(bytes / HBM peak, flops /
    TF32 peak); frac = T_roof / measured step time."""
    items = step_roofline_items(cfg, nnz, nnz_g)
    t_roof = 0.0
    t_hbm = 0.0
    t_tc = 0.0
    tot_b = tot_f = 0
    for _, count, nbytes, flops in items:
        tb = nbytes / (hbm_gbs * 1e9)
        tf = flops / (tf32_tflops * 1e12)
        t_roof += count * max(tb, tf)
        t_hbm += count * tb
        t_tc += count * tf
        tot_b += count * nbytes
        tot_f += count * flops
    return {"t_roof_ms": round(t_roof * 1e3, 4), "epoch_frac": round(t_roof * 1e3 / ms_per_step, 4),
            "step_bytes": int(tot_b), "step_tf32_flops": int(tot_f),
            "hbm_bound_ms": round(t_hbm * 1e3, 4), "tensor_bound_ms": round(t_tc * 1e3, 4),
            "kernels_modelled": len(items),
            "launches_modelled": int(sum(c for _, c, _, _ in items)),
            "peaks": {"hbm_gbs": hbm_gbs, "tf32_tflops": round(tf32_tflops, 1)}}


def load_traffic():
    if TRAFFIC_PATH.exists():
        try:
            return json.loads(TRAFFIC_PATH.read_text())
        except Exception:
            return {}
    return {}


class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap,"
             "timestamp")
    INTERVAL_MS = 20

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.path = None
        self.windows = []

    def start(self):
        """Start sampling and wait (up to 5 s) until the first sample is written,
        so that the timed region that follows is covered."""
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu_index), f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", str(self.INTERVAL_MS), "-f", self.path],
                stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
            return
        t0 = time.time()
        while time.time() - t0 < 5.0:
            try:
                if Path(self.path).stat().st_size > 0:
                    break
            except OSError:
                pass
            time.sleep(0.01)

    def begin(self):
        """Host time at the start of a timed region (pair with end())."""
        self.windows.append([time.time(), None])

    def end(self):
        if self.windows:
            self.windows[-1][1] = time.time()

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(2.0 * self.INTERVAL_MS / 1e3)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        try:
            lines = Path(self.path).read_text().splitlines()
        finally:
            try:
                os.unlink(self.path)
            except OSError:
                pass
        return self.summarize(self.in_windows(lines, self.windows))

    @staticmethod
    def in_windows(lines, windows):
        """The samples whose timestamp (last column, local time) falls inside one
        of the [begin, end] host-time windows; all samples when none carries a
        readable timestamp or no window was marked."""
        import datetime
        if not windows:
            return lines
        kept, stamped = [], 0
        for line in lines:
            parts = [p.strip() for p in line.split(",")]
            try:
                ts = datetime.datetime.strptime(parts[-1], "%Y/%m/%d %H:%M:%S.%f").timestamp()
            except (ValueError, IndexError):
                continue
            stamped += 1
            if any(b <= ts <= (e if e is not None else ts) for b, e in windows):
                kept.append(line)
        return kept if stamped else lines

    @staticmethod
    def summarize(lines):
        """{sm_mhz: median, sm_max_mhz, reasons: throttle reasons seen Active,
        samples} of `nvidia-smi --query-gpu=QUERY --format=csv,noheader,nounits`
        lines, or None without samples."""
        rows = []
        for line in lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------ workload
def build_graph(cfg, device):
    from cign_b200 import synth
    from cign_b200.graph_operator import (build_sparse_normalized_adjacency,
                                          prepare_fixed_csr_operator, prepare_gat_edge_index,
                                          to_graph_format)
    from cign_b200.multihop_csr_pipeline import prepare_multihop_csr_operator
    edge = synth.make_edges(cfg, device=device).to(device)
    n = cfg.num_nodes
    ei, adj = build_sparse_normalized_adjacency(edge, n)
    base = prepare_fixed_csr_operator(adj)
    op = prepare_multihop_csr_operator(base, dense_cols=2 * cfg.hidden_dim, powers=cfg.hops)
    gat_e = prepare_gat_edge_index(ei, n)
    (rp, c), (r, cp), perm = to_graph_format(gat_e.flip(0), n)
    return op, ((rp, c), (r, cp), perm), int(base.nnz), int(c.numel())


def build_model_and_data(cfg, device, seed=0, capturable=False):
    from cign_b200 import synth
    from cign_b200.model_cign import build_model
    torch.manual_seed(seed)
    x, y, train, _, _ = synth.make_features(cfg)
    model = build_model(in_dim=cfg.in_dim, hidden_dim=cfg.hidden_dim, out_dim=cfg.num_classes,
                        num_layers=cfg.layers, dropout=cfg.dropout, hop_scales=cfg.hops,
                        gat_heads=cfg.heads, gat_dropout=cfg.gat_dropout).to(device)
    opt = torch.optim.Adam(model.parameters(), lr=0.003, weight_decay=1e-5, capturable=capturable,
                           fused=True)
    return model, opt, x, y, train


def train_step(model, opt, op, x, y, train_idx):
    """optimizer.zero_grad -> forward -> CE(train rows) -> backward -> Adam.step (torch's
    fused Adam)
    (generic_engine/train_cign.py:2103-2148).  The train rows are gathered by
    a precomputed index (the same rows, in the same order, as the reference's
    boolean mask, without its host synchronisation)."""
    opt.zero_grad(set_to_none=True)
    logits = model(x, op)
    loss = F.cross_entropy(logits.index_select(0, train_idx), y.index_select(0, train_idx))
    loss.backward()
    opt.step()
    return loss


# ------------------------------------------------------------- kernel timing
def algorithmic_bytes(kind, N, nnz, F=0, H=0, C=0, K=0, D=0, nnz_g=0):
    """Compulsory HBM bytes of one launch (each tensor read/written once)."""
    if kind == "spmm":
        return 4 * (N + 1) + 8 * nnz + 8 * N * F
    if kind == "spmm_add":
        return 4 * (N + 1) + 8 * nnz + 12 * N * F
    if kind == "gat_fwd":
        return 4 * (N + 1) + 4 * nnz_g + 8 * N * H + 4 * N * H * C + 4 * C + 8 * N * C + 8 * N * H
    if kind == "gat_bwd":
        return (8 * (N + 1) + 12 * nnz_g + 8 * N * H + 4 * N * H * C + 8 * N * C + 8 * N * H
                + 4 * N * H * C + 8 * N * H + 4 * C)
    if kind == "gat_agg_fwd":
        return 4 * (N + 1) + 4 * nnz_g + 8 * N * H + 4 * N * D + 4 * N * H * D + 8 * N * H
    if kind == "gat_agg_bwd":
        return (8 * (N + 1) + 12 * nnz_g + 24 * N * H + 4 * N * D + 4 * N * H * D + 4 * N * C
                + 4 * N * H * C)
    if kind == "pack_proj":  # G written for the backward (keep_g)
        return (8 * N * D + 8 * K * N * D + 4 * N * K + 8 * K * N * D + 4 * C * 2 * K * D
                + 4 * N * C + 4 * C)
    if kind == "pack_fwd":
        return 8 * N * D + 8 * K * N * D + 4 * N * K + 8 * K * N * D
    if kind == "gate_pack_fwd":  # pack_fwd with alpha written instead of read, + gate W and b
        return 8 * N * D + 8 * K * N * D + 4 * N * K + 8 * K * N * D + 8 * K * D + 4 * K
    if kind == "pack_bwd":
        return 8 * K * N * D + 8 * N * D + 8 * K * N * D + 4 * N * K + 8 * N * D + 8 * K * N * D + 4 * N * K
    raise ValueError(kind)


def time_launches(fn, reps, stream):
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    fn()
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(reps):
        fn()
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end) / reps * 1e-3  # seconds per call


def kernel_breakdown(cfg, op, gat_graph, nnz, nnz_g, device, pack_proj_in_step=False):
    """Per-op device time (CUDA events on the launching stream) of the native
    kernels on the workload's own shapes, with launches per training step
    (0 for a kernel timed here that the step does not launch)."""
    from cign_b200 import _pack, collapsed_gat
    from cign_b200.plans import gat_plan_for
    N, D, H, K, L = cfg.num_nodes, cfg.hidden_dim, cfg.heads, len(cfg.hops), cfg.layers
    Fw = 2 * D
    stream = torch.cuda.current_stream(device)
    g = torch.Generator(device=device).manual_seed(1)
    plan = op.plan.spmm if hasattr(op, "plan") else op.native3.plan.spmm
    X = torch.randn(N, Fw, device=device, generator=g)
    G = torch.randn(N, Fw, device=device, generator=g)
    t_spmm = time_launches(lambda: plan.spmm(X), 20, stream)
    t_spmm_add = time_launches(lambda: plan.spmm(X, transpose=True, addend=G), 20, stream)
    (rp, c), (r, cp), perm = gat_graph
    gplan = gat_plan_for(rp, c, r, cp, perm)
    x = torch.randn(N, D, device=device, generator=g)
    a = torch.randn(N, H, device=device, generator=g)
    # the model's calls: the forward keeps the edge weights for the backward
    fwd = lambda: collapsed_gat.gat_agg_forward_keep_raw(gplan, a, a, x, H, 0.2,  # noqa: E731
                                                         cfg.gat_dropout, 7)
    t_gat_fwd = time_launches(fwd, 10, stream)
    z, emax, esum, wts = fwd()
    del z
    gz = torch.randn(N, H * D, device=device, generator=g)
    gpre = torch.randn(N, D, device=device, generator=g)
    t_gat_bwd = time_launches(lambda: collapsed_gat.gat_agg_backward_raw(
        gplan, a, a, x, emax, esum, gz, gpre, 0.2, cfg.gat_dropout, 7, wts=wts), 10, stream)
    del gz, gpre
    Hn = torch.randn(N, D, device=device, generator=g)
    Cn = torch.randn(N, D, device=device, generator=g)
    props = [torch.randn(N, 2 * D, device=device, generator=g) for _ in range(K)]
    alpha = torch.softmax(torch.randn(N, K, device=device, generator=g), -1)
    gw = torch.randn(K, 2 * D, device=device, generator=g) / (2 * D) ** 0.5
    gb = torch.zeros(K, device=device)
    t_pack_f = time_launches(lambda: _pack.gate_pack_forward(Hn, Cn, props, gw, gb, 1, 1, 0, 0), 20,
                             stream)
    go = torch.randn(N, 2 * K * D, device=device, generator=g)
    t_pack_b = time_launches(lambda: _pack.pack_backward(go, Hn, Cn, props, alpha, 1, 0, 0, True),
                             20, stream)
    del go
    Wp = torch.randn(D, 2 * K * D, device=device, generator=g) / (2 * K * D) ** 0.5
    bp = torch.zeros(D, device=device)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    t_pp = time_launches(lambda: _pack.pack_proj_forward(Hn, Cn, props, alpha, Wp, bp, True), 20,
                         stream)
    torch.backends.cuda.matmul.allow_tf32 = prev
    rows = {
        "spmm_fwd_hop": (t_spmm, L * K, algorithmic_bytes("spmm", N, nnz, F=Fw)),
        "spmm_bwd_hop_fused_add": (t_spmm_add, L * K, algorithmic_bytes("spmm_add", N, nnz, F=Fw)),
        "gat_agg_fwd": (t_gat_fwd, L, algorithmic_bytes("gat_agg_fwd", N, nnz, H=H, D=D,
                                                        nnz_g=nnz_g)),
        "gat_agg_bwd": (t_gat_bwd, L, algorithmic_bytes("gat_agg_bwd", N, nnz, H=H, C=D, D=D,
                                                        nnz_g=nnz_g)),
        "pack_proj_tcgen05_fwd": (t_pp, L if pack_proj_in_step else 0,
                                  algorithmic_bytes("pack_proj", N, nnz, K=K, D=D, C=D)),
        "gate_pack_fwd": (t_pack_f, L, algorithmic_bytes("gate_pack_fwd", N, nnz, K=K, D=D)),
        "pack_bwd": (t_pack_b, L, algorithmic_bytes("pack_bwd", N, nnz, K=K, D=D)),
    }
    out = {}
    for name, (t, per_step, nbytes) in rows.items():
        out[name] = {"ms_per_launch": round(t * 1e3, 4), "launches_per_step": per_step,
                     "ms_per_step": round(t * per_step * 1e3, 4),
                     "algorithmic_bytes": int(nbytes),
                     "achieved_gbs": round(nbytes / t / 1e9, 1)}
    if not pack_proj_in_step:
        out["pack_proj_tcgen05_fwd"]["note"] = ("not launched by this step: with G_raw kept for "
                                                "the backward the pack kernel + cuBLAS run instead")
    return out


def hop_roofline(timer, N, nnz, peak, peak_kind, with_traffic=True):
    """Roofline of the dominant kernel, the k-hop SpMM (spmm_rows_kernel plus its
    hub-row combine; the largest share of the step's device time), from the
    CUDA events recorded around every k-hop call inside the timed steps."""
    t_ms = 0.0
    launches = 0
    alg = 0
    mix = {"fwd": 0, "bwd_add": 0, "bwd": 0}
    F = None
    for kind, n_hops, n_add, F, start, end, rows, rec_nnz in timer.records:
        t_ms += start.elapsed_time(end)
        launches += n_hops
        if kind == "fwd":
            mix["fwd"] += n_hops
        else:
            mix["bwd_add"] += n_add
            mix["bwd"] += n_hops - n_add
        Nr = N if rows is None else rows
        Zr = nnz if rec_nnz is None else rec_nnz
        alg += (n_hops - n_add) * algorithmic_bytes("spmm", Nr, Zr, F=F)
        alg += n_add * algorithmic_bytes("spmm_add", Nr, Zr, F=F)
    if launches == 0:
        return None
    per_launch_s = t_ms * 1e-3 / launches
    achieved = alg / launches / per_launch_s / 1e9
    tr = load_traffic().get("spmm_hop", {}) if with_traffic else {}
    traffic = None
    if all(k in tr for k in ("fwd", "bwd_add", "bwd")):
        traffic = int((mix["fwd"] * tr["fwd"] + mix["bwd_add"] * tr["bwd_add"]
                       + mix["bwd"] * tr["bwd"]) / launches)
    return {"bound": "hbm", "kernel": "spmm_hop (spmm_rows_kernel + hub combine), F=%d" % F,
            "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "traffic": traffic,
            "algorithmic_bytes": int(alg / launches), "ms_per_launch": round(per_launch_s * 1e3, 4),
            "launches_timed": launches, "launch_mix": mix,
            "gather_bytes": int(4 * nnz * F),
            "timing": "CUDA events around every k-hop call in the timed steps, on the launching stream"}


# ------------------------------------------------------- partitioned (N > 1)
def run_partitioned(args, cfg, metric, world, rank, local_rank, device):
    """cfg2 (the default) scales weakly: a power-law graph of world x cfg2
    size (same generator, degree law and per-node widths) is row-partitioned
    over the ranks, so each rank trains a cfg2-sized row range.  Other
    workloads (e.g. cfg4, the 2.45M-node RMAT graph) scale strongly: the
    same graph is partitioned over more ranks.  Halo rows move once per hop
    and per GAT layer; parameter gradients are summed with one all-reduce
    per step."""
    from dataclasses import replace

    import torch.distributed as dist

    from cign_b200 import _lib, synth
    from cign_b200.distributed import allreduce_gradients, partition_graph
    from cign_b200.graph_operator import (build_sparse_normalized_adjacency,
                                          prepare_fixed_csr_operator, prepare_gat_edge_index,
                                          to_graph_format)
    from cign_b200.model_cign import build_model

    torch.backends.cuda.matmul.allow_tf32 = True
    lib = _lib.load_library()
    weak = args.workload == "cfg2"
    gcfg = (replace(cfg, name=f"{cfg.name}_x{world}", num_nodes=cfg.num_nodes * world,
                    num_edges=cfg.num_edges * world) if weak else cfg)
    n = gcfg.num_nodes
    edge = synth.make_edges(gcfg, device=device).to(device)
    ei, adj = build_sparse_normalized_adjacency(edge, n)
    base = prepare_fixed_csr_operator(adj)
    (rp, c), _, _ = to_graph_format(prepare_gat_edge_index(ei, n).flip(0), n)
    bounds, hplan, exch, dop, dgat = partition_graph(
        base.csr, rp, c, world, rank, device,
        transport={"nccl": None, "peer": "peer", "peer-copy": "peer-copy"}[args.exchange])
    r0, r1 = bounds[rank], bounds[rank + 1]
    nnz = int(base.nnz)
    x_all, y_all, train_all, _, _ = synth.make_features(gcfg)
    torch.manual_seed(0)  # identical parameters on every rank
    model = build_model(in_dim=cfg.in_dim, hidden_dim=cfg.hidden_dim, out_dim=cfg.num_classes,
                        num_layers=cfg.layers, dropout=cfg.dropout, hop_scales=cfg.hops,
                        gat_heads=cfg.heads, gat_dropout=cfg.gat_dropout).to(device)
    model.prepare_fused_gat_graph(dgat)
    torch.manual_seed(1000 + rank)  # independent dropout streams per rank
    use_graph = not args.eager
    opt = torch.optim.Adam(model.parameters(), lr=0.003, weight_decay=1e-5, capturable=use_graph,
                           fused=True)
    x_cpu = x_all[r0:r1].contiguous()
    x = x_cpu.to(device)
    y = y_all[r0:r1].to(device)
    train_global = int(train_all.sum())
    mine = train_all[r0:r1].nonzero().squeeze(1).to(device)
    edge_passes = 2 * cfg.layers * len(cfg.hops) * nnz  # whole graph, all ranks
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)
    params = list(model.parameters())

    def step(xin):
        exch.begin_step()
        opt.zero_grad(set_to_none=True)
        logits = model(xin, dop)
        loss = F.cross_entropy(logits.index_select(0, mine), y.index_select(0, mine),
                               reduction="sum") / train_global
        loss.backward()
        allreduce_gradients(params)
        opt.step()
        return loss

    from cign_b200.plans import HopTimer, SpmmPlan
    hop_timer = HopTimer()
    graphed = None
    if use_graph:
        from cign_b200.graph_step import GraphedStep

        def install_timer():  # the captured step records its local SpMM events
            SpmmPlan.hop_timer = hop_timer

        graphed = GraphedStep(lambda: step(x), device, warmup=args.warmup,
                              before_capture=install_timer)
        SpmmPlan.hop_timer = None
        run_step = lambda xin: graphed()  # noqa: E731  (x is the graph's static input)
    else:
        for _ in range(args.warmup):
            step(x)
        run_step = step
    torch.cuda.synchronize()
    launches_before = int(lib.cign_kernel_launches())
    stream = torch.cuda.current_stream(device)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    sampler = ClockSampler(local_rank)
    dist.barrier()
    torch.cuda.synchronize()
    push_timer = []
    if not use_graph:
        SpmmPlan.hop_timer = hop_timer  # events around every local row-block SpMM
        if hasattr(exch, "timer"):
            exch.timer = push_timer  # events around every halo push + its barrier
    sampler.start()
    sampler.begin()
    for i in range(args.steps):
        flush.zero_()
        starts[i].record(stream)
        run_step(x)
        ends[i].record(stream)
    torch.cuda.synchronize()
    sampler.end()
    SpmmPlan.hop_timer = None
    if hasattr(exch, "timer"):
        exch.timer = None
    # per rank: push-kernel ms, barrier-wait ms, bytes sent (per step)
    push_mine = torch.tensor([sum(a.elapsed_time(b) for a, b, _, _ in push_timer) / args.steps,
                              sum(b.elapsed_time(c) for _, b, c, _ in push_timer) / args.steps,
                              sum(nb for _, _, _, nb in push_timer) / args.steps],
                             device=device, dtype=torch.float64)
    per_rank = [torch.empty_like(push_mine) for _ in range(world)]
    dist.all_gather(per_rank, push_mine)
    push_stats = [t.tolist() for t in per_rank] if push_timer else None
    clocks = sampler.stop()
    launches = (graphed.native_launches * args.steps if use_graph
                else int(lib.cign_kernel_launches()) - launches_before)
    step_ms = [a.elapsed_time(b) for a, b in zip(starts, ends)]
    total_s = sum(step_ms) * 1e-3
    t = torch.tensor([total_s], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_s = float(t.item())

    x_pin = x_cpu.pin_memory()
    dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        x.copy_(x_pin, non_blocking=True)
        loss_host = float(run_step(x).item())
    e1.record(stream)
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) * 1e-3], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_s = float(t.item())
    halo = torch.tensor([hplan.n_halo], device=device, dtype=torch.float64)
    halo_max = halo.clone()
    dist.all_reduce(halo)
    dist.all_reduce(halo_max, op=dist.ReduceOp.MAX)
    if graphed is not None:
        del graphed  # release the graph (it holds collectives) before the buffers go
        torch.cuda.synchronize()
    if hasattr(exch, "close"):
        exch.close()
    if rank == 0:
        peak, peak_kind = load_peaks()
        result = {
            "metric": metric,
            "value": round(edge_passes * args.steps / total_s / 1e9, 4), "unit": "GTEPS",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(total_s / args.steps * 1e3, 4), "higher_is_better": True,
            "scaling": "weak" if weak else "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": gcfg.name, "nodes": n, "directed_edges": gcfg.num_edges,
                       "nnz_P": nnz, "nodes_per_gpu": n // world, "in_dim": cfg.in_dim,
                       "hidden": cfg.hidden_dim, "hops": list(cfg.hops), "heads": cfg.heads,
                       "layers": cfg.layers, "dropout": cfg.dropout,
                       "parallelism": f"row-partition x{world}",
                       "exchange": ("halo rows per hop and per GAT layer: " +
                                    {"nccl": "NCCL point-to-point",
                                     "peer": "stored into the peers' IPC-mapped buffers over "
                                             "NVLink by SM stores (cign_halo_push)",
                                     "peer-copy": "copied into the peers' IPC-mapped buffers "
                                                  "over NVLink by the copy engines "
                                                  "(cign_halo_push_copy)"}[args.exchange] +
                                    "; one gradient all-reduce per step"),
                       "halo_rows_total": int(halo.item()),
                       "halo_rows_max_per_rank": int(halo_max.item()),
                       "l2": "flushed between timed steps (256 MiB write)",
                       "launch": "one CUDA graph per step" if use_graph else "eager"},
            "e2e": {"value": round(edge_passes * args.steps / e2e_s / 1e9, 4), "unit": "GTEPS",
                    "h2d_bytes_per_step": int(x_cpu.numel() * 4), "d2h_bytes_per_step": 4,
                    "ms_per_step": round(e2e_s / args.steps * 1e3, 4)},
            "gpu_launches": launches,
            "step_ms_rank0": [round(v, 3) for v in step_ms],
            "halo_push_per_rank": (None if push_stats is None else {
                "push_ms_per_step": [round(v[0], 2) for v in push_stats],
                "barrier_wait_ms_per_step": [round(v[1], 2) for v in push_stats],
                "bytes_sent_per_step": [int(v[2]) for v in push_stats],
                "push_gbs": [round(v[2] / max(v[0], 1e-9) * 1e-6, 1) for v in push_stats],
                "timing": "CUDA events around each halo push kernel (push) and its ordering "
                          "all-reduce (barrier wait: includes waiting for slower ranks); the "
                          "k-hop pushes run on a side stream beside the own-column SpMM"}),
            "roofline": hop_roofline(hop_timer, hplan.n_own, dop.nnz_local, peak, peak_kind,
                                     with_traffic=False),
            "cpu_baseline": None, "clocks": clocks,
            "final_loss": round(loss_host, 5),
        }
        print(json.dumps(result), flush=True)
    dist.barrier()
    return 0


# ------------------------------------------------------------------ sweep
def sweep_bf16(device, emit):
    """fp32 against bf16 feature storage (fp32 accumulation) for the two
    gathers of the path -- one k-hop SpMM hop at F = 1024 and the
    aggregate-first GAT forward at D = 512 -- on the cfg2 graph and on one
    eighth of the cfg5 graph (an RMAT graph of 1.25M nodes and 40M edges,
    the row block one of 8 GPUs owns, with the same degree law), each run
    as a square operator.  Device times from CUDA events."""
    from cign_b200 import collapsed_gat, synth
    from cign_b200.graph_operator import (build_sparse_normalized_adjacency,
                                          prepare_fixed_csr_operator, prepare_gat_edge_index,
                                          to_graph_format)
    from cign_b200.multihop_csr_pipeline import _csr_parts_int32
    from cign_b200.plans import SpmmPlan, gat_plan_for
    stream = torch.cuda.current_stream(device)
    g = torch.Generator(device=device).manual_seed(5)
    cfg5 = synth.CONFIGS["cfg5"]
    graphs = [("cfg2_powerlaw24492", lambda: synth.make_edges(synth.CONFIGS["cfg2"]).to(device),
               synth.CONFIGS["cfg2"].num_nodes),
              ("cfg5_rmat_shard1250000", lambda: synth.rmat_graph(
                  cfg5.num_nodes // 8, cfg5.num_edges // 8, seed=cfg5.seed, device=device).to(device),
               cfg5.num_nodes // 8)]
    for name, make, n in graphs:
        edge = make()
        ei, adj = build_sparse_normalized_adjacency(edge, n)
        base = prepare_fixed_csr_operator(adj)
        plan = SpmmPlan(*_csr_parts_int32(base.csr))
        nnz = int(base.nnz)
        del adj
        F = 1024
        X = torch.randn(n, F, device=device, generator=g)
        Xb = X.to(torch.bfloat16)
        t32 = time_launches(lambda: plan.spmm(X), 5, stream)
        t16 = time_launches(lambda: plan.spmm_bf16(Xb, torch.bfloat16), 5, stream)
        emit({"op": "spmm_hop_storage", "storage_graph": name, "storage_nodes": n,
              "storage_nnz_P": nnz, "F": F,
              "fp32_ms": round(t32 * 1e3, 4), "bf16_ms": round(t16 * 1e3, 4),
              "gather_tbs_fp32": round(4 * nnz * F / t32 / 1e12, 2),
              "gather_tbs_bf16": round(2 * nnz * F / t16 / 1e12, 2)})
        del X, Xb
        (rp, c), (r, cp), perm = to_graph_format(prepare_gat_edge_index(ei, n).flip(0), n)
        gplan = gat_plan_for(rp, c, r, cp, perm)
        H, D = 8, 512
        x = torch.randn(n, D, device=device, generator=g)
        xb = x.to(torch.bfloat16)
        a = torch.randn(n, H, device=device, generator=g)
        t32 = time_launches(lambda: collapsed_gat.gat_agg_forward_raw(gplan, a, a, x, H, 0.2, 0.5, 7),
                            3, stream)
        t16 = time_launches(lambda: collapsed_gat.gat_agg_forward_raw(gplan, a, a, xb, H, 0.2, 0.5,
                                                                      7), 3, stream)
        emit({"op": "gat_agg_fwd_storage", "storage_graph": name, "storage_nodes": n,
              "storage_nnz_gat": int(c.numel()),
              "heads": H, "D": D, "fp32_ms": round(t32 * 1e3, 4), "bf16_ms": round(t16 * 1e3, 4)})
        del x, xb, gplan, plan, base, ei, edge
        torch.cuda.empty_cache()


def run_sweep(args, device):
    """isolated kernel sweep on the cfg2 graph.  One JSON line per
    case: k-hop SpMM (hops 1..8, F in {64, 128, 512}; forward chain and its
    transposed backward) next to cuSPARSE (torch.sparse.mm, the library the
    reference's MultiHopCsrPlan calls); the collapsed GAT layer with 1/4/8
    heads (aggregate-first form, forward + backward, and the drop-in form);
    the Clifford pack and its proj mix GEMM at 8 and 16 blades with the
    contraction in TF32 and in FP32.  Device times from CUDA events."""
    from cign_b200 import _pack, collapsed_gat, synth
    from cign_b200.plans import gat_plan_for
    cfg = synth.CONFIGS["cfg2"]
    op, gat_graph, nnz, nnz_g = build_graph(cfg, device)
    plan = op.plan.spmm
    N = cfg.num_nodes
    stream = torch.cuda.current_stream(device)
    g = torch.Generator(device=device).manual_seed(3)
    csr = op.base.csr if hasattr(op, "base") else None

    def emit(d):
        d.update({"sweep": "configs[2]", "graph": cfg.name, "nodes": N, "nnz_P": nnz})
        print(json.dumps(d), flush=True)

    ops = set(args.sweep_ops.split(",")) if args.sweep_ops else {"spmm", "gat", "pack"}
    if "bf16" in ops:
        sweep_bf16(device, emit)
    for F in ((64, 128, 512) if "spmm" in ops else ()):
        X = torch.randn(N, F, device=device, generator=g)
        for K in range(1, 9):
            t_f = time_launches(lambda: plan.forward(X, K), 5, stream)
            gs = [torch.randn(N, F, device=device, generator=g) for _ in range(K)]
            t_b = time_launches(lambda: plan.backward(gs, F), 5, stream)
            line = {"op": "multihop_spmm", "F": F, "hops": K,
                    "fwd_ms": round(t_f * 1e3, 4), "bwd_ms": round(t_b * 1e3, 4),
                    "gteps": round(2 * K * nnz / (t_f + t_b) / 1e9, 3)}
            if csr is not None:
                def cus():
                    y = X
                    for _ in range(K):
                        y = torch.sparse.mm(csr, y)
                    return y
                line["cusparse_fwd_ms"] = round(time_launches(cus, 5, stream) * 1e3, 4)
            emit(line)
    (rp, c), (r, cp), perm = gat_graph
    gplan = gat_plan_for(rp, c, r, cp, perm)
    D = cfg.hidden_dim
    for H in ((1, 4, 8) if "gat" in ops else ()):
        x = torch.randn(N, D, device=device, generator=g)
        a = torch.randn(N, H, device=device, generator=g)
        z, emax, esum = collapsed_gat.gat_agg_forward_raw(gplan, a, a, x, H, 0.2, 0.5, 7)
        U = torch.randn(N, H * D, device=device, generator=g)
        gp = torch.randn(N, D, device=device, generator=g)
        t_af = time_launches(lambda: collapsed_gat.gat_agg_forward_raw(gplan, a, a, x, H, 0.2, 0.5, 7),
                             5, stream)
        t_ab = time_launches(lambda: collapsed_gat.gat_agg_backward_raw(
            gplan, a, a, x, emax, esum, U, gp, 0.2, 0.5, 7), 5, stream)
        xin = torch.randn(N, H, D, device=device, generator=g)
        bias = torch.zeros(D, device=device)
        t_cf = time_launches(lambda: collapsed_gat.gat_forward_raw(gplan, a, a, xin, bias, 0.2, 0.5, 7),
                             5, stream)
        out, pre, em2, es2 = collapsed_gat.gat_forward_raw(gplan, a, a, xin, bias, 0.2, 0.5, 7)
        t_cb = time_launches(lambda: collapsed_gat.gat_backward_raw(
            gplan, a, a, xin, pre, em2, es2, gp, 0.2, 0.5, 7), 5, stream)
        emit({"op": "collapsed_gat", "heads": H, "channels": D,
              "aggregate_first_fwd_ms": round(t_af * 1e3, 4),
              "aggregate_first_bwd_ms": round(t_ab * 1e3, 4),
              "drop_in_fwd_ms": round(t_cf * 1e3, 4), "drop_in_bwd_ms": round(t_cb * 1e3, 4)})
    K = 3
    for blades in ((8, 16) if "pack" in ops else ()):
        Dp = 64 * blades
        Hn = torch.randn(N, Dp, device=device, generator=g)
        Cn = torch.randn(N, Dp, device=device, generator=g)
        props = [torch.randn(N, 2 * Dp, device=device, generator=g) for _ in range(K)]
        alpha = torch.softmax(torch.randn(N, K, device=device, generator=g), -1)
        W = torch.randn(Dp, 2 * K * Dp, device=device, generator=g) / (2 * K * Dp) ** 0.5
        t_pf = time_launches(lambda: _pack.pack_forward(Hn, Cn, props, alpha, 1, 0, 0), 5, stream)
        G = _pack.pack_forward(Hn, Cn, props, alpha, 1, 0, 0)
        line = {"op": "clifford_pack_mix", "blades": blades, "D": Dp, "hops": K,
                "pack_fwd_ms": round(t_pf * 1e3, 4)}
        for name, tf32 in (("tf32", True), ("fp32", False)):
            prev = torch.backends.cuda.matmul.allow_tf32
            torch.backends.cuda.matmul.allow_tf32 = tf32
            t_mm = time_launches(lambda: G.mm(W.t()), 5, stream)
            torch.backends.cuda.matmul.allow_tf32 = prev
            line[f"mix_{name}_ms"] = round(t_mm * 1e3, 4)
            line[f"mix_{name}_tflops"] = round(2 * N * 2 * K * Dp * Dp / t_mm / 1e12, 1)
        if _pack.pack_proj_supported(Dp, K, Dp):
            # pack + mix as one tcgen05 GEMM with the pack as its A-operand prologue
            bias = torch.zeros(Dp, device=device)
            for keep in (False, True):
                t_pp = time_launches(lambda: _pack.pack_proj_forward(
                    Hn, Cn, props, alpha, W, bias, keep), 5, stream)
                key = "pack_mix_tcgen05" + ("_with_g" if keep else "")
                line[f"{key}_ms"] = round(t_pp * 1e3, 4)
                line[f"{key}_tflops"] = round(2 * N * 2 * K * Dp * Dp / t_pp / 1e12, 1)
        emit(line)
    return 0


# ------------------------------------------------------------------ CPU arm
def cpu_sample_config(cfg, sample_nodes):
    """The CPU arm's bounded sample of a workload: the same generator and
    average degree on min(sample_nodes, N) nodes (the whole workload when it
    is that small already)."""
    from dataclasses import replace
    if sample_nodes >= cfg.num_nodes:
        return cfg
    scale = sample_nodes / cfg.num_nodes
    return replace(cfg, name=cfg.name + f"_sample{sample_nodes}", num_nodes=sample_nodes,
                   num_edges=int(round(cfg.num_edges * scale)))


def run_cpu_oracle(cfg, steps, warmup, budget_s=None):
    """The reference's torch path restated in oracle/ (CPU, all host threads)
    on one sampled graph of the workload's family; returns (GTEPS, s/step)."""
    from cign_b200 import synth
    from oracle import graph as og
    from oracle import ops
    from oracle.model import OracleCIGN
    torch.set_num_threads(os.cpu_count() or 1)
    edge = synth.make_edges(cfg).numpy()
    n = cfg.num_nodes
    r, c, v = og.normalized_adjacency(edge, n)
    P = ops.csr_tensor(*og.csr_of(r, c, v, n), n, n)
    nnz = int(v.size)
    gat_graph = og.gat_graph(og.prepare_gat_edge_index(og.to_undirected(edge, n), n), n)
    torch.manual_seed(0)
    x, y, train, _, _ = synth.make_features(cfg)
    model = OracleCIGN(cfg.in_dim, cfg.hidden_dim, cfg.num_classes, cfg.layers, cfg.hops,
                       cfg.dropout, cfg.heads, cfg.gat_dropout)
    opt = torch.optim.Adam(model.parameters(), lr=0.003, weight_decay=1e-5)

    def step():
        opt.zero_grad()
        logits = model(x, P, P, gat_graph, initial_seed=0)
        loss = F.cross_entropy(logits[train], y[train])
        loss.backward()
        opt.step()

    for _ in range(warmup):
        step()
    times = []
    t_all = time.perf_counter()
    for _ in range(steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
        if budget_s is not None and time.perf_counter() - t_all > budget_s:
            break
    t = statistics.median(times)
    edge_passes = 2 * cfg.layers * len(cfg.hops) * nnz
    return edge_passes / t / 1e9, t, len(times), nnz


# ------------------------------------------------------------------ main
def main():
    ap = argparse.ArgumentParser(description="CIGN B200 training-step benchmark")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="cfg2")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-sample-nodes", type=int, default=0,
                    help="nodes of the CPU arms' graph (0: the whole workload graph)")
    ap.add_argument("--cpu-budget-s", type=float, default=240.0,
                    help="the reference arm stops timing after this many seconds")
    ap.add_argument("--sweep", action="store_true",
                    help="configs[2] isolated kernel sweep (one JSON line per case) instead of "
                         "the training-step benchmark")
    ap.add_argument("--pack-proj", choices=["auto", "fused", "separate"], default="auto",
                    help="block pack + proj: tcgen05 pack-prologue GEMM (fused), pack kernel + "
                         "cuBLAS (separate), or fused only when G_raw is recomputed (auto)")
    ap.add_argument("--sweep-ops", default="",
                    help="comma-separated subset of the sweep: spmm,gat,pack (default all), "
                         "bf16 (fp32 against bf16 feature storage, cfg2 and a cfg5 shard)")
    ap.add_argument("--layers", type=int, default=0,
                    help="override the workload's number of CIGN blocks (0: the config's)")
    ap.add_argument("--exchange", choices=["peer", "peer-copy", "nccl"], default="peer",
                    help="halo exchange of the multi-GPU run")
    ap.add_argument("--eager", action="store_true",
                    help="launch every op from Python each step (default: replay one CUDA graph)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    from cign_b200 import synth
    cfg = synth.CONFIGS[args.workload]
    if args.layers > 0:
        from dataclasses import replace as dc_replace
        cfg = dc_replace(cfg, layers=args.layers)
    metric = "CIGN fwd+bwd train-step GTEPS (SpMM edge-passes/s)"
    from cign_b200 import block_fused
    block_fused.USE_TCGEN05_PACK_PROJ = {"auto": None, "fused": True,
                                         "separate": False}[args.pack_proj]
    if cfg.num_nodes > GRAPH_CAPTURE_MAX_NODES:
        # launch overhead is negligible at this size, and a captured step would
        # hold a second copy of the activations in the graph's private pool
        args.eager = True

    if args.impl == "reference":
        # CPU reference arm: rank 0 only; other ranks exit without work.
        if rank != 0:
            return 0
        sample = cpu_sample_config(cfg, args.cpu_sample_nodes or cfg.num_nodes)
        gteps, t, done, nnz = run_cpu_oracle(sample, max(1, args.steps), 1,
                                             budget_s=args.cpu_budget_s)
        cores = os.cpu_count() or 1
        line = {
            "impl": "reference", "metric": metric, "value": round(gteps, 6), "unit": "GTEPS",
            "n_gpus": args.gpus, "steps": done, "warmup": 1, "ms_per_step": round(t * 1e3, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": sample.name, "nodes": sample.num_nodes, "nnz_P": nnz,
                       "hidden": cfg.hidden_dim, "hops": list(cfg.hops), "heads": cfg.heads,
                       "layers": cfg.layers, "dropout": cfg.dropout,
                       "note": "the reference's torch training step on the host CPU "
                               "(oracle/ restatement, all host threads)"},
            "cpu_baseline": {"value": round(gteps, 6), "unit": "GTEPS", "cores": cores,
                             "kind": "port",
                             "sample": f"{done} full training step(s) (median) on the whole "
                                       f"{sample.name} graph (N={sample.num_nodes}, nnz={nnz})"},
            "e2e": {"value": round(gteps, 6), "unit": "GTEPS", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line), flush=True)
        return 0

    if not torch.cuda.is_available():
        raise SystemExit("bench.py (impl ours) needs a CUDA GPU")
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=device)
        try:
            return run_partitioned(args, cfg, metric, world, rank, local_rank, device)
        finally:
            dist.destroy_process_group()
    torch.backends.cuda.matmul.allow_tf32 = True
    torch.backends.cudnn.allow_tf32 = True

    from cign_b200 import _lib
    lib = _lib.load_library()
    if args.sweep:
        return run_sweep(args, device)

    op, gat_graph, nnz, nnz_g = build_graph(cfg, device)
    use_graph = not args.eager
    model, opt, x_cpu, y_cpu, train_cpu = build_model_and_data(cfg, device, seed=rank,
                                                               capturable=use_graph)
    x = x_cpu.to(device)
    y = y_cpu.to(device)
    train_idx = train_cpu.to(device).nonzero().squeeze(1)
    model.prepare_fused_gat_graph(gat_graph)
    edge_passes = 2 * cfg.layers * len(cfg.hops) * nnz
    # GAT edge passes: per layer one forward pass and three backward passes
    # (edge logits, softmax backward, transposed aggregation) over nnz_g x H
    gat_edge_passes = cfg.layers * nnz_g * cfg.heads * 4
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device)

    from cign_b200.plans import HopTimer, SpmmPlan
    hop_timer = HopTimer()
    step = lambda: train_step(model, opt, op, x, y, train_idx)  # noqa: E731
    graphed = None
    if use_graph:
        from cign_b200.graph_step import GraphedStep

        def install_timer():  # the captured step records its k-hop events
            SpmmPlan.hop_timer = hop_timer

        graphed = GraphedStep(step, device, warmup=args.warmup, before_capture=install_timer)
        SpmmPlan.hop_timer = None
        run_step = graphed
    else:
        for _ in range(args.warmup):
            step()
        run_step = step
    torch.cuda.synchronize()
    launches_before = int(lib.cign_kernel_launches())

    stream = torch.cuda.current_stream(device)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    sampler = ClockSampler(local_rank)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    if not use_graph:
        SpmmPlan.hop_timer = hop_timer  # CUDA events around every k-hop call, same stream
    sampler.start()
    sampler.begin()
    for i in range(args.steps):
        flush.zero_()  # L2 flush between timed steps (outside the per-step events)
        starts[i].record(stream)
        run_step()
        ends[i].record(stream)
    torch.cuda.synchronize()
    sampler.end()
    SpmmPlan.hop_timer = None
    # kernels launched per step: counted by the library while the graph was
    # captured (one step), or over the timed eager steps
    timed_launches = (graphed.native_launches * args.steps if use_graph
                      else int(lib.cign_kernel_launches()) - launches_before)
    if dist is not None:
        dist.barrier()
    step_s = [s.elapsed_time(e) * 1e-3 for s, e in zip(starts, ends)]
    total_s = sum(step_s)
    if dist is not None:
        t = torch.tensor([total_s], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_s = float(t.item())
    ms_per_step = total_s / args.steps * 1e3
    value = edge_passes * world * args.steps / total_s / 1e9

    # end-to-end through the public API: every step's features are copied
    # from pinned host memory (on a copy stream, one step ahead, into a
    # double-buffered staging tensor, then into the step's input buffer) and
    # every step's loss is copied back to pinned host memory; all of it
    # inside the timed region.
    x_pin = x_cpu.pin_memory()
    copy_stream = torch.cuda.Stream(device)
    staging = [torch.empty_like(x), torch.empty_like(x)]
    copied = [torch.cuda.Event(), torch.cuda.Event()]
    consumed = [torch.cuda.Event(), torch.cuda.Event()]
    loss_pin = torch.empty(args.steps, dtype=torch.float32).pin_memory()
    e_start = torch.cuda.Event(enable_timing=True)
    e_end = torch.cuda.Event(enable_timing=True)

    def stage(i):  # H2D copy of step i's input on the copy stream
        b = i % 2
        with torch.cuda.stream(copy_stream):
            if i >= 2:
                copy_stream.wait_event(consumed[b])
            staging[b].copy_(x_pin, non_blocking=True)
            copied[b].record(copy_stream)

    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    sampler.begin()
    e_start.record(stream)
    copy_stream.wait_event(e_start)
    stage(0)
    for i in range(args.steps):
        b = i % 2
        stream.wait_event(copied[b])
        x.copy_(staging[b])
        consumed[b].record(stream)
        if i + 1 < args.steps:
            stage(i + 1)
        loss = run_step()
        loss_pin[i:i + 1].copy_(loss.detach().reshape(1), non_blocking=True)  # D2H of the result
    e_end.record(stream)
    torch.cuda.synchronize()
    sampler.end()
    clocks = sampler.stop()  # samples inside the two timed regions
    loss_host = float(loss_pin[-1])
    e2e_s = e_start.elapsed_time(e_end) * 1e-3
    if dist is not None:
        t = torch.tensor([e2e_s], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
        dist.barrier()
    e2e_value = edge_passes * world * args.steps / e2e_s / 1e9

    result = None
    if rank == 0:
        peak, peak_kind = load_peaks()
        blk = model.blocks[0]
        keep_g = not blk._recompute_pack(torch.empty(cfg.num_nodes, 0))
        pp_in_step = ((not keep_g) if block_fused.USE_TCGEN05_PACK_PROJ is None
                      else bool(block_fused.USE_TCGEN05_PACK_PROJ))
        kernels = (kernel_breakdown(cfg, op, gat_graph, nnz, nnz_g, device, pp_in_step)
                   if cfg.num_nodes <= GRAPH_CAPTURE_MAX_NODES else None)
        roofline = hop_roofline(hop_timer, cfg.num_nodes, nnz, peak, peak_kind)
        tf32_peak, tf32_kind = load_tf32_peak()
        step_roof = step_roofline(cfg, nnz, nnz_g, ms_per_step, peak, tf32_peak)
        step_roof["peaks"]["kind"] = f"HBM {peak_kind}; TF32 {tf32_kind}"
        if roofline is not None:
            roofline["epoch_frac"] = step_roof["epoch_frac"]
            roofline["epoch"] = step_roof
        if roofline is not None and use_graph:
            roofline["timing"] = ("CUDA events captured around every k-hop call inside the step "
                                  "graph, read after the last timed replay")
        cpu_baseline = None
        if world == 1 and not args.no_cpu_baseline:
            sample = cpu_sample_config(cfg, args.cpu_sample_nodes or cfg.num_nodes)
            gteps_cpu, t_cpu, done, nnz_s = run_cpu_oracle(sample, 3, 1, budget_s=60.0)
            cpu_baseline = {"value": round(gteps_cpu, 6), "unit": "GTEPS",
                            "cores": os.cpu_count() or 1, "kind": "port",
                            "sample": f"{done} full training step(s) (median) of the oracle "
                                      f"model on the whole {sample.name} graph "
                                      f"(N={sample.num_nodes}, nnz={nnz_s})",
                            "s_per_step": round(t_cpu, 3)}
        result = {
            "metric": metric, "value": round(value, 4), "unit": "GTEPS", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": cfg.name, "nodes": cfg.num_nodes, "directed_edges": cfg.num_edges,
                       "nnz_P": nnz, "nnz_gat": nnz_g, "in_dim": cfg.in_dim,
                       "hidden": cfg.hidden_dim, "channels_x_blades": "64x8", "hops": list(cfg.hops),
                       "heads": cfg.heads, "layers": cfg.layers, "dropout": cfg.dropout,
                       "dense_gemm": "tf32 (cuBLAS via torch)",
                       "pack_proj": args.pack_proj,
                       "l2": "flushed between timed steps (256 MiB write)",
                       "launch": "one CUDA graph per step" if use_graph else "eager",
                       "parallelism": f"replicas{world}" if world > 1 else "single"},
            "epoch_ms": round(ms_per_step, 4),
            "gat_gteps": round(gat_edge_passes * world * args.steps / total_s / 1e9, 4),
            "gat_edge_passes_per_step": int(gat_edge_passes * world),
            "ms_per_step_median": round(statistics.median(step_s) * 1e3, 4),
            "e2e": {"value": round(e2e_value, 4), "unit": "GTEPS",
                    "h2d_bytes_per_step": int(x.numel() * 4), "d2h_bytes_per_step": 4,
                    "ms_per_step": round(e2e_s / args.steps * 1e3, 4),
                    "pipeline": "H2D of step i+1 overlaps step i (copy stream); loss D2H "
                                "into pinned memory every step"},
            "gpu_launches": timed_launches,
            "roofline": roofline,
            "kernels": kernels,
            "cpu_baseline": cpu_baseline,
            "clocks": clocks,
            "final_loss": round(loss_host, 5),
        }
        print(json.dumps(result), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
