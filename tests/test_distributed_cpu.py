"""Host logic of the row-partitioned path, on the CPU: partition balance,
halo bookkeeping (what each rank sends equals what its peers expect), and the
halo exchange forward/backward over torch.distributed (gloo, 2 and 3 ranks
as processes on 127.0.0.1), checked against the global tensors."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cign_b200 import distributed, synth
from cign_b200.distributed import (DistMultiHop, HaloExchange, HaloPlan, _local_block,
                                   halo_gather, partition_rows)
from cign_b200.graph_operator import build_sparse_normalized_adjacency


def _global_csr(n=700, e=5000, seed=3):
    edge = synth.powerlaw_graph(n, e, seed=seed)
    _, adj = build_sparse_normalized_adjacency(edge, n)
    return adj.coalesce().to_sparse_csr()


@pytest.mark.parametrize("row_weight", [1, 30])
def test_partition_balances_rows_plus_nnz(row_weight):
    """Ranges balance row_weight * rows + non-zeros to within one row's work."""
    P = _global_csr()
    crow = P.crow_indices()
    n, nnz = crow.numel() - 1, int(crow[-1])
    total = row_weight * n + nnz
    for world in (1, 2, 3, 8):
        b = partition_rows(crow, world, row_weight)
        assert b[0] == 0 and b[-1] == n and all(x <= y for x, y in zip(b, b[1:]))
        work = [row_weight * (b[r + 1] - b[r]) + int(crow[b[r + 1]] - crow[b[r]])
                for r in range(world)]
        assert sum(work) == total
        assert max(work) <= total / world + int((crow[1:] - crow[:-1]).max()) + row_weight


def test_halo_plans_agree_between_ranks():
    P = _global_csr()
    crow, col = P.crow_indices(), P.col_indices()
    for world in (2, 3, 5):
        b = partition_rows(crow, world)
        plans = [HaloPlan(crow, col, b, r) for r in range(world)]
        for r in range(world):
            for p in range(world):
                if p == r:
                    continue
                # what r sends to p is exactly p's halo rows owned by r, in p's order
                sent = plans[r].send_idx[p] + plans[r].r0
                owned = plans[p].halo[(plans[p].halo >= plans[r].r0) & (plans[p].halo < plans[r].r1)]
                assert torch.equal(sent, owned)
                assert plans[r].send_counts[p] == plans[p].recv_counts[r]
        # the local blocks, with the halo filled in, reproduce P @ X row by row
        X = torch.randn(P.size(0), 6)
        Y = P @ X
        for r in range(world):
            pl = plans[r]
            lcrow, lcol, lval = _local_block(crow, col, P.values(), pl)
            x_ext = torch.cat([X[pl.r0:pl.r1], X[pl.halo]])
            blk = torch.sparse_csr_tensor(lcrow, lcol, lval, (pl.n_own, pl.n_own + pl.n_halo))
            assert torch.allclose(blk @ x_ext, Y[pl.r0:pl.r1], atol=1e-6)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _exchange_worker(rank, world, port, errors):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        P = _global_csr()
        crow, col = P.crow_indices(), P.col_indices()
        b = partition_rows(crow, world)
        plans = [HaloPlan(crow, col, b, r) for r in range(world)]
        me = plans[rank]
        ex = HaloExchange(me, "cpu")
        X = torch.randn(P.size(0), 5, generator=torch.Generator().manual_seed(11))
        x_own = X[me.r0:me.r1].clone().requires_grad_(True)
        x_ext = halo_gather(x_own, ex)
        assert torch.equal(x_ext.detach(), torch.cat([X[me.r0:me.r1], X[me.halo]]))
        # backward: every rank weights its extended rows with its own G
        Gs = [torch.randn(p.n_own + p.n_halo, 5, generator=torch.Generator().manual_seed(100 + r))
              for r, p in enumerate(plans)]
        (x_ext * Gs[rank]).sum().backward()
        want = torch.zeros(P.size(0), 5)
        for r, p in enumerate(plans):
            want[p.r0:p.r1] += Gs[r][:p.n_own]
            want.index_add_(0, p.halo, Gs[r][p.n_own:])
        assert torch.allclose(x_own.grad, want[me.r0:me.r1], atol=1e-6)
        # the split hop's path: halo rows only, gradients returned to owners
        halo, ev = ex.gather_halo(X[me.r0:me.r1].contiguous())
        assert ev is None and torch.equal(halo, X[me.halo])
        recv, _ = ex.return_halo(Gs[rank][me.n_own:])
        g_own = Gs[rank][:me.n_own].clone()
        ex.add_returned(g_own, recv)
        assert torch.allclose(g_own, want[me.r0:me.r1], atol=1e-6)
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # pragma: no cover - reported to the parent
        errors.put(f"rank {rank}: {exc!r}")
        raise


@pytest.mark.parametrize("world", [2, 3])
def test_halo_exchange_gloo(world):
    ctx = mp.get_context("spawn")
    errors = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, world, port, errors)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    for p in procs:
        if p.is_alive():
            p.kill()
    msgs = []
    while not errors.empty():
        msgs.append(errors.get())
    assert not msgs, msgs
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


class _CpuPlan:
    """CPU stand-in for the native SpmmPlan of a partitioned block (the
    host logic around it is what these tests cover)."""

    def __init__(self, rows, cols, vals, n_rows, n_cols, dev):
        self.A = torch.sparse_coo_tensor(torch.stack([rows, cols]), vals,
                                         (n_rows, n_cols)).coalesce()

    def spmm(self, x, transpose=False, addend=None):
        y = torch.sparse.mm(self.A.t() if transpose else self.A, x)
        return y if addend is None else y + addend


class _RecordingExchange(HaloExchange):
    """The base exchange, recording the sequence of exchange steps."""

    def __init__(self, plan):
        super().__init__(plan, "cpu")
        self.calls = []

    def gather_halo(self, x_own):
        self.calls.append("gather_halo")
        return super().gather_halo(x_own)

    def return_halo(self, g_halo):
        self.calls.append("return_halo")
        return super().return_halo(g_halo)

    def add_returned(self, g_own, recv):
        self.calls.append("add_returned")
        super().add_returned(g_own, recv)


def _two_component_csr():
    """Nodes 0-399 and 400-599 form two unconnected graphs."""
    a = synth.powerlaw_graph(400, 3000, seed=4)
    b = synth.powerlaw_graph(200, 1500, seed=5) + 400
    _, adj = build_sparse_normalized_adjacency(torch.cat([a, b], dim=1), 600)
    return adj.coalesce().to_sparse_csr()


def _khop_worker(rank, world, port, errors):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        distributed._csr_plan = _CpuPlan  # CPU stand-in for the native plans
        P = _two_component_csr()
        bounds = [0, 200, 400, 600]  # rank 2 owns the second graph: no halo columns
        me = HaloPlan(P.crow_indices(), P.col_indices(), bounds, rank)
        assert (me.n_halo == 0) == (rank == 2)
        ex = _RecordingExchange(me)
        hop = DistMultiHop(P, me, ex)
        gen = torch.Generator().manual_seed(21)
        X = torch.randn(600, 4, generator=gen)
        Gs = {p: torch.randn(600, 4, generator=gen) for p in (1, 2, 3)}
        x_own = X[me.r0:me.r1].clone().requires_grad_(True)
        outs = hop.powers(x_own, (1, 2, 3))
        loss = sum((outs[p] * Gs[p][me.r0:me.r1]).sum() for p in (1, 2, 3))
        loss.backward()
        Y, want_grad, Pt = X, torch.zeros(600, 4), P.t()
        for p in (1, 2, 3):
            Y = P @ Y
            assert torch.allclose(outs[p].detach(), Y[me.r0:me.r1], atol=1e-5), p
            g = Gs[p]
            for _ in range(p):
                g = Pt @ g
            want_grad += g
        assert torch.allclose(x_own.grad, want_grad[me.r0:me.r1], atol=1e-5)
        # the raw forward/backward pair the fused block node calls
        ys = hop.forward(X[me.r0:me.r1].contiguous(), 3)
        Y = X
        for p in (1, 2, 3):
            Y = P @ Y
            assert torch.allclose(ys[p - 1], Y[me.r0:me.r1], atol=1e-5), p
        gx = hop.backward([Gs[p][me.r0:me.r1].contiguous() for p in (1, 2, 3)], 4)
        assert torch.allclose(gx, want_grad[me.r0:me.r1], atol=1e-5)
        # every rank took the same exchange steps in the same order
        seqs = [None] * world
        dist.all_gather_object(seqs, ex.calls)
        assert all(q == seqs[0] for q in seqs), seqs
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # pragma: no cover - reported to the parent
        errors.put(f"rank {rank}: {exc!r}")
        raise


def test_partitioned_khop_with_a_halo_free_rank_gloo():
    """k-hop forward and backward over three ranks, one of which has no halo
    columns, in the autograd form and as the raw forward/backward pair:
    results equal the global P^p X and its gradient, and all ranks
    take the same sequence of exchange steps (one collective each on the
    peer-memory transport)."""
    ctx = mp.get_context("spawn")
    errors = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_khop_worker, args=(r, 3, port, errors)) for r in range(3)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    for p in procs:
        if p.is_alive():
            p.kill()
    msgs = []
    while not errors.empty():
        msgs.append(errors.get())
    assert not msgs, msgs
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]

def test_interleaved_push_order():
    """The push order visits the per-peer blocks round-robin from the given
    peer and is a permutation of the whole send list."""
    counts = [3, 0, 2, 4]
    order = distributed.interleaved_order(counts, first=2)
    assert order.tolist() == [3, 5, 0, 4, 6, 1, 7, 2, 8]
    g = torch.Generator().manual_seed(5)
    for w in (2, 3, 8):
        for first in range(w):
            counts = torch.randint(0, 50, (w,), generator=g).tolist()
            order = distributed.interleaved_order(counts, first)
            assert sorted(order.tolist()) == list(range(sum(counts)))
