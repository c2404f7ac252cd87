"""A CIGN training step captured in one CUDA graph (GraphedStep) replays the
eager step: the same losses and parameters over consecutive steps, the native
dropout ops drawing the same per-call seeds from the device seed table as the
eager host counters would give."""
import copy

import pytest
import torch
import torch.nn.functional as F

from cign_b200 import seeds, synth
from cign_b200.graph_operator import (build_sparse_normalized_adjacency,
                                      prepare_fixed_csr_operator, prepare_gat_edge_index,
                                      to_graph_format)
from cign_b200.graph_step import GraphedStep
from cign_b200.model_cign import build_model
from cign_b200.multihop_csr_pipeline import prepare_multihop_csr_operator

pytestmark = pytest.mark.gpu


def _setup(dev, n=600, e=5000, in_dim=32, hidden=64, classes=5):
    edge = synth.powerlaw_graph(n, e, seed=3).to(dev)
    ei, adj = build_sparse_normalized_adjacency(edge, n)
    op = prepare_multihop_csr_operator(prepare_fixed_csr_operator(adj), dense_cols=2 * hidden)
    (rp, c), (r, cp), perm = to_graph_format(prepare_gat_edge_index(ei, n).flip(0), n)
    torch.manual_seed(0)
    model = build_model(in_dim=in_dim, hidden_dim=hidden, out_dim=classes, num_layers=2,
                        dropout=0.5, hop_scales=(1, 2, 3), gat_heads=2, gat_dropout=0.5).to(dev)
    model.prepare_fused_gat_graph(((rp, c), (r, cp), perm))
    model.dropout = 0.0  # net-level torch dropout off: only the native ops draw seeds
    x = torch.randn(n, in_dim, device=dev)
    y = torch.randint(0, classes, (n,), device=dev)
    idx = torch.arange(0, n, 2, device=dev)
    return model, op, x, y, idx


def _stepper(model, op, x, y, idx):
    opt = torch.optim.Adam(model.parameters(), lr=0.01, capturable=True)

    def step():
        opt.zero_grad(set_to_none=True)
        loss = F.cross_entropy(model(x, op).index_select(0, idx), y.index_select(0, idx))
        loss.backward()
        opt.step()
        return loss
    return step


def test_graphed_step_replays_eager_steps(cuda):
    model0, op, x, y, idx = _setup(cuda)
    model_a = copy.deepcopy(model0)
    model_b = copy.deepcopy(model0)
    step_a = _stepper(model_a, op, x, y, idx)
    step_b = _stepper(model_b, op, x, y, idx)

    seeds.set_host_counters(100, 200)
    eager = [float(step_a()) for _ in range(6)]
    counters_after_eager = seeds.host_counters()

    seeds.set_host_counters(100, 200)
    g = GraphedStep(step_b, cuda, warmup=3)
    replayed = [float(g()) for _ in range(3)]
    g.finish()
    for i, (a, b) in enumerate(zip(eager[3:], replayed)):
        assert abs(a - b) <= 1e-6 * max(1.0, abs(a)), f"step {i + 4}: eager {a} graph {b}"
    for (name, pa), (_, pb) in zip(model_a.named_parameters(), model_b.named_parameters()):
        err = float((pa - pb).abs().max())
        assert err <= 1e-5 * max(1.0, float(pa.abs().max())), f"{name}: max diff {err}"
    assert seeds.host_counters() == counters_after_eager


def test_seed_table_matches_host_stream(cuda):
    table = seeds.DeviceSeedTable(cuda)
    seeds.set_host_counters(7, 11)
    table.counters.copy_(torch.tensor([7, 11]))
    with table.recording():
        slots = [seeds.next_seed(seeds.GAT, 0.3), seeds.next_seed(seeds.BLOCK, 0.3, 1),
                 seeds.next_seed(seeds.BLOCK, 0.0, 2), seeds.next_seed(seeds.BLOCK, 0.5, 2),
                 seeds.next_seed(seeds.GAT, 0.5)]
    assert slots[2] == 0  # p == 0: seed 0, no slot, no counter advance
    for step in range(2):
        table.advance()
        got = [int(s.item()) for s in (slots[0], slots[1], slots[3], slots[4])]
        want = [seeds.next_seed(seeds.GAT, 0.3), seeds.next_seed(seeds.BLOCK, 0.3, 1),
                seeds.next_seed(seeds.BLOCK, 0.5, 2), seeds.next_seed(seeds.GAT, 0.5)]
        assert got == want, f"step {step}"
    table.sync_host_counters(prefetched=False)
    assert table.counters.tolist() == list(seeds.host_counters())
