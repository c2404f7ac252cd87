"""The row-partitioned CIGN step on the GPU kernels (rectangular SpMM and GAT
plans, halo exchange) against the unpartitioned model: logits row by row and
parameter gradients summed over ranks.  The ranks run as 2 or 3 processes
sharing one GPU, exchanging halo rows through host memory over gloo (waits
are host-side only), so the test needs a single GPU."""
import copy
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, errors):
    try:
        from cign_b200 import synth
        from cign_b200.distributed import StagedGlooP2P, partition_graph
        from cign_b200.graph_operator import (build_sparse_normalized_adjacency,
                                              prepare_fixed_csr_operator, prepare_gat_edge_index,
                                              to_graph_format)
        from cign_b200.model_cign import build_model
        from cign_b200.multihop_csr_pipeline import prepare_multihop_csr_operator
        from tests.helpers import assert_parity

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        torch.backends.cuda.matmul.allow_tf32 = False
        n, in_dim, hidden, classes = 900, 32, 64, 5
        edge = synth.powerlaw_graph(n, 7000, seed=5).to(dev)
        ei, adj = build_sparse_normalized_adjacency(edge, n)
        base = prepare_fixed_csr_operator(adj)
        (rp, c), (r, cp), perm = to_graph_format(prepare_gat_edge_index(ei, n).flip(0), n)
        torch.manual_seed(0)
        model0 = build_model(in_dim=in_dim, hidden_dim=hidden, out_dim=classes, num_layers=2,
                             dropout=0.0, hop_scales=(1, 2, 3), gat_heads=2,
                             gat_dropout=0.0).to(dev)
        g = torch.Generator().manual_seed(1)
        x = torch.randn(n, in_dim, generator=g).to(dev)
        y = torch.randint(0, classes, (n,), generator=g).to(dev)
        train = torch.arange(0, n, 3, device=dev)

        # unpartitioned reference (every rank computes it)
        ref = copy.deepcopy(model0)
        ref.prepare_fused_gat_graph(((rp, c), (r, cp), perm))
        op = prepare_multihop_csr_operator(base, dense_cols=2 * hidden)
        logits_ref = ref(x, op)
        F.cross_entropy(logits_ref[train], y[train], reduction="sum").div(train.numel()).backward()

        # partitioned
        bounds, plan, ex, dop, dgat = partition_graph(base.csr, rp, c, world, rank, dev,
                                                      StagedGlooP2P())
        part = copy.deepcopy(model0)
        part.prepare_fused_gat_graph(dgat)
        r0, r1 = bounds[rank], bounds[rank + 1]
        logits = part(x[r0:r1].contiguous(), dop)
        mine = train[(train >= r0) & (train < r1)] - r0
        loss = F.cross_entropy(logits[mine], y[r0:r1][mine], reduction="sum") / train.numel()
        loss.backward()
        assert_parity(logits.detach(), logits_ref.detach()[r0:r1], what=f"logits rank {rank}")
        for (name, p_ref), (_, p) in zip(ref.named_parameters(), part.named_parameters()):
            gsum = p.grad.detach().cpu()
            dist.all_reduce(gsum)
            assert_parity(gsum, p_ref.grad.detach().cpu(), what=f"grad {name}")
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # pragma: no cover - reported to the parent
        errors.put(f"rank {rank}: {exc!r}")
        raise


@pytest.mark.parametrize("world", [2, 3])
def test_partitioned_model_matches_unpartitioned(cuda, world):
    ctx = mp.get_context("spawn")
    errors = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, errors)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    msgs = []
    while not errors.empty():
        msgs.append(errors.get())
    assert not msgs, msgs
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
