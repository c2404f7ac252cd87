"""Host-side logic that needs no GPU: dropout seed streams, shape gates of
the fused kernels, the graph-capture policy of the bench.

The seed formulas are restated from the reference (collapsed_gat.py:204-211
for GAT calls, fused_block_ops.py:46-50 for block-op calls) and checked
against cign_b200.seeds, including the rule that p == 0 calls neither get a
seed nor advance the stream."""
import pytest
import torch

from cign_b200 import _pack, seeds
from cign_b200.jk_norm import jk_norm_supported

MASK63 = (1 << 63) - 1


def reference_gat_seed(base, call_id):
    return (base + 0x9E3779B97F4A7C15 * (call_id + 1)) & MASK63


def reference_block_seed(base, call_1based, tag):
    return (base + 0x9E3779B97F4A7C15 * call_1based + 0xD2B74407B1CE6E93 * int(tag)) & MASK63


@pytest.fixture()
def fresh_counters():
    saved = seeds.host_counters()
    seeds.set_host_counters(0, 0)
    yield
    seeds.set_host_counters(*saved)


def test_seed_streams_follow_reference_formulas(fresh_counters):
    torch.manual_seed(1234567)
    base = int(torch.initial_seed()) & MASK63
    got_gat = [seeds.next_seed(seeds.GAT, 0.3) for _ in range(3)]
    assert got_gat == [reference_gat_seed(base, c) for c in range(3)]
    got_block = [seeds.next_seed(seeds.BLOCK, 0.5, tag) for tag in (1, 2, 1)]
    assert got_block == [reference_block_seed(base, c + 1, t)
                         for c, t in zip(range(3), (1, 2, 1))]


def test_zero_probability_does_not_advance(fresh_counters):
    torch.manual_seed(7)
    base = int(torch.initial_seed()) & MASK63
    assert seeds.next_seed(seeds.GAT, 0.0) == 0
    assert seeds.next_seed(seeds.BLOCK, 0.0, 3) == 0
    assert seeds.host_counters() == (0, 0)
    assert seeds.next_seed(seeds.GAT, 0.1) == reference_gat_seed(base, 0)


@pytest.mark.parametrize("D,K,dout,ok", [(512, 3, 512, True), (32, 1, 32, True),
                                         (48, 2, 64, False), (512, 9, 512, False),
                                         (512, 3, 1024, False), (512, 3, 48, False)])
def test_pack_proj_shape_gate(D, K, dout, ok):
    assert _pack.pack_proj_supported(D, K, dout) is ok


def test_jk_norm_gate_needs_cuda_fp32_equal_widths():
    cpu = [torch.zeros(4, 8) for _ in range(3)]
    assert not jk_norm_supported(cpu)  # CPU tensors: the torch path is used
    assert not jk_norm_supported([])


def test_graph_capture_policy():
    import bench
    from cign_b200 import synth
    assert synth.CONFIGS["cfg2"].num_nodes <= bench.GRAPH_CAPTURE_MAX_NODES
    assert synth.CONFIGS["cfg4"].num_nodes > bench.GRAPH_CAPTURE_MAX_NODES


def test_algorithmic_bytes_at_cfg2_shapes():
    """Roofline numerators (compulsory HBM bytes per launch: every tensor read
    or written once) at cfg2's shapes, N=24,492, nnz=390,042, D=512, F=2D,
    H=4, K=3."""
    import bench
    N, nnz, D, H, K = 24492, 390042, 512, 4, 3
    F = 2 * D
    ab = bench.algorithmic_bytes
    # SpMM pass: crow, col + val, X read, Y written (+ the fused addend)
    assert ab("spmm", N, nnz, F=F) == 4 * (N + 1) + 8 * nnz + 8 * N * F == 203_856_772
    assert ab("spmm_add", N, nnz, F=F) == 304_176_004
    assert ab("gat_agg_fwd", N, nnz, H=H, D=D, nnz_g=nnz) == 254_023_708
    assert ab("gat_agg_bwd", N, nnz, H=H, D=D, C=D, nnz_g=nnz) == 508_823_840
    assert ab("pack_fwd", N, nnz, D=D, K=K) == 702_528_528
    assert ab("pack_bwd", N, nnz, D=D, K=K) == 1_104_099_360
    assert ab("pack_proj", N, nnz, D=D, K=K, C=D) == 758_981_648
    with pytest.raises(ValueError):
        ab("unknown", N, nnz)


def test_clock_summary_of_nvidia_smi_samples():
    """The bench's clock record from `nvidia-smi --query-gpu` CSV lines (a
    fake sample: no GPU, no NVML): median SM clock under load, the max clock,
    and every throttle reason seen Active."""
    import bench
    lines = [
        "0, 1965, 1965, 650.1, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active",
        "0, 1800, 1965, 990.3, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
        "0, 1845, 1965, 995.0, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
        "garbage line",
    ]
    got = bench.ClockSampler.summarize(lines)
    assert got == {"sm_mhz": 1845.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"],
                   "samples": 3}
    hot = lines[:1] + ["0, 1200, 1965, 700.0, 0x48, Active, Not Active, Active, Not Active"]
    assert bench.ClockSampler.summarize(hot)["reasons"] == ["hw_slowdown", "sw_thermal_slowdown"]
    assert bench.ClockSampler.summarize([]) is None


def test_clock_samples_inside_timed_windows():
    """Only samples stamped inside a marked [begin, end] window count; lines
    without a timestamp keep the old behaviour (all samples)."""
    import datetime

    import bench

    def stamp(t):
        return datetime.datetime.fromtimestamp(t).strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]
    base = 1_800_000_000.0
    lines = [f"0, {mhz}, 1965, 900.0, 0x0, Not Active, Not Active, Not Active, Not Active, "
             f"{stamp(base + dt)}" for mhz, dt in ((345, 0.0), (1965, 1.0), (1950, 1.1), (345, 3.0))]
    kept = bench.ClockSampler.in_windows(lines, [[base + 0.5, base + 1.5]])
    assert bench.ClockSampler.summarize(kept) == {"sm_mhz": 1957.5, "sm_max_mhz": 1965.0,
                                                  "reasons": [], "samples": 2}
    unstamped = [ln.rsplit(",", 1)[0] for ln in lines]
    assert bench.ClockSampler.in_windows(unstamped, [[base, base + 1]]) == unstamped


def test_hop_roofline_from_recorded_events():
    """The bench's `roofline` object from k-hop timer records (fake CUDA
    events): algorithmic bytes per launch over the measured time per launch."""
    import bench

    class _Ev:
        def __init__(self, ms):
            self.ms = ms

        def elapsed_time(self, end):
            return end.ms - self.ms

    class _Timer:
        records = [("fwd", 3, 0, 1024, _Ev(0.0), _Ev(0.6), None, None),
                   ("bwd", 3, 2, 1024, _Ev(1.0), _Ev(1.9), None, None)]

    N, nnz, F = 24492, 390042, 1024
    r = bench.hop_roofline(_Timer(), N, nnz, 6449.7, "measured", with_traffic=False)
    alg = 4 * bench.algorithmic_bytes("spmm", N, nnz, F=F) + 2 * bench.algorithmic_bytes(
        "spmm_add", N, nnz, F=F)
    assert r["launches_timed"] == 6 and r["launch_mix"] == {"fwd": 3, "bwd_add": 2, "bwd": 1}
    assert r["algorithmic_bytes"] == int(alg / 6)
    assert abs(r["ms_per_launch"] - 1.5 / 6) < 1e-9
    assert abs(r["achieved"] - alg / 1.5e-3 / 1e9) < 0.1
    assert abs(r["frac"] - r["achieved"] / 6449.7) < 1e-4
    assert r["traffic"] is None and r["bound"] == "hbm" and r["unit"] == "GB/s"
    assert bench.hop_roofline(type("T", (), {"records": []})(), N, nnz, 1.0, "x") is None


def test_cpu_sample_is_never_larger_than_the_workload():
    import bench
    from cign_b200 import synth
    cfg1, cfg2 = synth.CONFIGS["cfg1"], synth.CONFIGS["cfg2"]
    assert bench.cpu_sample_config(cfg1, 6000) is cfg1
    s = bench.cpu_sample_config(cfg2, 6000)
    assert s.num_nodes == 6000 and s.name == "cfg2_powerlaw24492_sample6000"
    assert s.num_edges == round(cfg2.num_edges * 6000 / cfg2.num_nodes)
    assert (s.hidden_dim, s.hops, s.heads, s.layers) == (cfg2.hidden_dim, cfg2.hops, cfg2.heads,
                                                         cfg2.layers)


def test_step_roofline_model_at_cfg2():
    """The whole-step roofline: every modelled kernel counted once per launch,
    T_roof = sum of max(bytes / HBM, flops / TF32) and frac = T_roof / step."""
    import bench
    from cign_b200 import synth
    cfg = synth.CONFIGS["cfg2"]
    items = bench.step_roofline_items(cfg, 390042, 390042)
    names = [n for n, _, _, _ in items]
    assert len(names) == len(set(names))
    counts = dict((n, c) for n, c, _, _ in items)
    assert counts["k-hop SpMM fwd hop"] == 6
    assert counts["k-hop SpMM bwd hop (+g fused)"] + counts["k-hop SpMM bwd hop"] == 6
    flops = dict((n, f) for n, _, _, f in items)
    N, D, K = 24492, 512, 3
    assert flops["proj (GEMM)"] == 2 * N * D * 2 * K * D
    r = bench.step_roofline(cfg, 390042, 390042, 10.0, 6452.5, 700.0)
    manual = sum(c * max(b / 6452.5e9, f / 700e12) for _, c, b, f in items) * 1e3
    assert abs(r["t_roof_ms"] - round(manual, 4)) < 1e-3
    assert abs(r["epoch_frac"] - round(manual / 10.0, 4)) < 1e-4
    assert r["hbm_bound_ms"] <= r["t_roof_ms"] <= r["hbm_bound_ms"] + r["tensor_bound_ms"]


def test_block_node_gate():
    """The whole-block node takes CUDA fp32 inputs on an unpartitioned GAT
    graph only; CPU tensors, a partitioned graph (an object with a halo
    exchange) or a non-production pack switch fall back to the op-by-op
    block."""
    from cign_b200.block_node import block_node_applies
    from cign_b200.model_cign import GraphCliffordBlock

    block = GraphCliffordBlock(64, (1, 2, 3), gat_heads=2)
    H = torch.zeros(10, 64)
    triple = ((None, None), (None, None), None)
    assert not block_node_applies(block, H, object(), triple)  # CPU tensor

    class _Partitioned:
        halo = None

    class _FakeCuda:
        is_cuda = True
        dtype = torch.float32

        def dim(self):
            return 2

        def size(self, i):
            return (10, 64)[i]

    assert not block_node_applies(block, _FakeCuda(), object(), _Partitioned())
    block.interaction_mode = "old"
    assert not block_node_applies(block, _FakeCuda(), object(), triple)
