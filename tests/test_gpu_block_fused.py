"""The fused propagation/hop-gate/pack node (block_fused), with and without
the proj layer folded in, against the
op-by-op composition of the same block (multihop_csr_pipeline, hop_gate and
pack modules with autograd accumulating the gradients), on the full model."""
import copy

import pytest
import torch
import torch.nn.functional as F

import cign_b200.model_cign as mc
from cign_b200 import synth
from cign_b200.graph_operator import (build_sparse_normalized_adjacency,
                                      prepare_fixed_csr_operator, prepare_gat_edge_index,
                                      to_graph_format)
from cign_b200.multihop_csr_pipeline import prepare_multihop_csr_operator
from tests.helpers import assert_parity

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("block_node", [False, True])
@pytest.mark.parametrize("recompute", [False, True])
@pytest.mark.parametrize("hops,score", [((1, 2, 3), "new"), ((1, 3), "old"), ((2,), "new")])
def test_fused_block_matches_op_by_op(cuda, monkeypatch, hops, score, recompute, block_node):
    """recompute=True runs the node that also applies proj and recomputes
    G_raw in the backward instead of keeping it; block_node=True runs the
    whole block as one node (block_node.cign_block: in-kernel gradient
    accumulation), block_node=False the fused propagate/gate/pack/proj node
    inside the op-by-op block."""
    torch.backends.cuda.matmul.allow_tf32 = False
    n, in_dim, hidden = 800, 24, 64
    edge = synth.powerlaw_graph(n, 6000, seed=2).to(cuda)
    ei, adj = build_sparse_normalized_adjacency(edge, n)
    op = prepare_multihop_csr_operator(prepare_fixed_csr_operator(adj), dense_cols=2 * hidden,
                                       powers=hops)
    gat = to_graph_format(prepare_gat_edge_index(ei, n).flip(0), n)
    torch.manual_seed(0)
    model = mc.build_model(in_dim=in_dim, hidden_dim=hidden, out_dim=4, num_layers=2,
                           dropout=0.0, hop_scales=hops, gat_heads=2, gat_dropout=0.0,
                           alpha_score_mode=score).to(cuda)
    model.prepare_fused_gat_graph(gat)
    other = copy.deepcopy(model)
    for block in model.blocks:
        block.recompute_pack = recompute
        block.use_block_node = block_node
    x = torch.randn(n, in_dim, device=cuda)
    y = torch.randint(0, 4, (n,), device=cuda)
    out = model(x, op)
    F.cross_entropy(out, y).backward()
    monkeypatch.setattr(mc, "native_spmm_plan", lambda operator: None)
    ref = other(x, op)
    F.cross_entropy(ref, y).backward()
    assert_parity(out.detach(), ref.detach(), what="logits")
    for (name, p), (_, q) in zip(model.named_parameters(), other.named_parameters()):
        assert_parity(p.grad, q.grad, what=f"grad {name}")


def test_tcgen05_pack_proj_in_model(cuda, monkeypatch):
    """With TF32 matmuls on, the block's pack + proj runs on the tcgen05
    pack-prologue GEMM; it must agree with the pack kernel + cuBLAS TF32 proj
    within the TF32 contraction tolerance, for G kept and recomputed."""
    import cign_b200.block_fused as bf
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        n, in_dim, hidden, hops = 900, 24, 64, (1, 2, 3)
        edge = synth.powerlaw_graph(n, 7000, seed=5).to(cuda)
        ei, adj = build_sparse_normalized_adjacency(edge, n)
        op = prepare_multihop_csr_operator(prepare_fixed_csr_operator(adj),
                                           dense_cols=2 * hidden, powers=hops)
        gat = to_graph_format(prepare_gat_edge_index(ei, n).flip(0), n)
        torch.manual_seed(0)
        model = mc.build_model(in_dim=in_dim, hidden_dim=hidden, out_dim=4, num_layers=2,
                               dropout=0.0, hop_scales=hops, gat_heads=2,
                               gat_dropout=0.0).to(cuda)
        model.prepare_fused_gat_graph(gat)
        x = torch.randn(n, in_dim, device=cuda)
        y = torch.randint(0, 4, (n,), device=cuda)

        def run(use_tcgen05, recompute):
            m = copy.deepcopy(model)
            for block in m.blocks:
                block.recompute_pack = recompute
            monkeypatch.setattr(bf, "USE_TCGEN05_PACK_PROJ", use_tcgen05)
            out = m(x, op)
            F.cross_entropy(out, y).backward()
            return out.detach(), [p.grad for p in m.parameters()]

        ref_out, ref_grads = run(False, False)
        for recompute in (False, True):
            out, grads = run(True, recompute)
            assert_parity(out, ref_out, tol=2e-3, atol=1e-4, what="logits")
            for (name, _), g, r in zip(model.named_parameters(), grads, ref_grads):
                assert_parity(g, r, tol=2e-3, atol=1e-4, what=f"grad {name}")
    finally:
        torch.backends.cuda.matmul.allow_tf32 = False


def test_block_node_with_dropout_matches_op_by_op(cuda):
    """The whole-block node against the op-by-op block with every dropout on
    (block dropout 0.5, attention dropout 0.3): the same seed draws in the
    same order, so the same masks, logits and gradients."""
    from cign_b200 import seeds
    torch.backends.cuda.matmul.allow_tf32 = False
    n, in_dim, hidden, hops = 700, 20, 64, (1, 2, 3)
    edge = synth.powerlaw_graph(n, 5000, seed=9).to(cuda)
    ei, adj = build_sparse_normalized_adjacency(edge, n)
    op = prepare_multihop_csr_operator(prepare_fixed_csr_operator(adj), dense_cols=2 * hidden,
                                       powers=hops)
    gat = to_graph_format(prepare_gat_edge_index(ei, n).flip(0), n)
    torch.manual_seed(0)
    model = mc.build_model(in_dim=in_dim, hidden_dim=hidden, out_dim=4, num_layers=2,
                           dropout=0.5, hop_scales=hops, gat_heads=2, gat_dropout=0.3).to(cuda)
    model.prepare_fused_gat_graph(gat)
    other = copy.deepcopy(model)
    for block in other.blocks:
        block.use_block_node = False
    x = torch.randn(n, in_dim, device=cuda)
    y = torch.randint(0, 4, (n,), device=cuda)
    counters = seeds.host_counters()
    torch.manual_seed(1)  # the net's torch dropout on x and on the JK output
    out = model(x, op)
    F.cross_entropy(out, y).backward()
    seeds.set_host_counters(*counters)
    torch.manual_seed(1)
    ref = other(x, op)
    F.cross_entropy(ref, y).backward()
    assert_parity(out.detach(), ref.detach(), what="logits")
    for (name, p), (_, q) in zip(model.named_parameters(), other.named_parameters()):
        assert_parity(p.grad, q.grad, what=f"grad {name}")
