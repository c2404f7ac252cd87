"""PeerHaloExchange (halo rows stored into the peers' IPC-mapped buffers by
cign_halo_push, or copied there by the copy engines with
cign_halo_push_copy) against the NCCL point-to-point exchange: the same extended
tensors forward and the same gathered gradients backward, and the same
halo rows / returned gradients through the asynchronous halo-only path
(side-stream pushes), over three steps (buffers reused per step).  Needs 2
GPUs; skipped otherwise."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, errors, copy):
    try:
        from cign_b200 import synth
        from cign_b200.distributed import (HaloExchange, HaloPlan, PeerHaloExchange, halo_gather,
                                           partition_rows)
        from cign_b200.graph_operator import build_sparse_normalized_adjacency

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
        n = 3000
        _, adj = build_sparse_normalized_adjacency(synth.powerlaw_graph(n, 20000, seed=4), n)
        P = adj.coalesce().to_sparse_csr()
        crow, col = P.crow_indices(), P.col_indices()
        b = partition_rows(crow, world)
        plan = HaloPlan(crow, col, b, rank)
        ref = HaloExchange(plan, dev)
        peer = PeerHaloExchange(plan, dev, copy=copy)
        for step in range(3):
            peer.begin_step()
            for F in (64, 1024):
                g = torch.Generator(device=dev).manual_seed(100 * step + F + rank)
                x = torch.randn(plan.n_own, F, device=dev, generator=g)
                xr = x.clone().requires_grad_(True)
                xp = x.clone().requires_grad_(True)
                er = halo_gather(xr, ref)
                ep = halo_gather(xp, peer)
                assert torch.equal(er.detach(), ep.detach()), f"gather F={F} step={step}"
                w = torch.randn(er.shape, device=dev, generator=g)
                (er * w).sum().backward()
                (ep * w).sum().backward()
                assert torch.equal(xr.grad, xp.grad), f"scatter F={F} step={step}"
                # halo rows only, pushed on the side stream (the split hop's path)
                hr, _ = ref.gather_halo(x)
                hp, ev = peer.gather_halo(x)
                torch.cuda.current_stream(dev).wait_event(ev)
                assert torch.equal(hr, hp), f"gather_halo F={F} step={step}"
                gh = torch.randn(plan.n_halo, F, device=dev, generator=g)
                rr, _ = ref.return_halo(gh)
                rp, ev = peer.return_halo(gh)
                torch.cuda.current_stream(dev).wait_event(ev)
                a, c = x.clone(), x.clone()
                ref.add_returned(a, rr)
                peer.add_returned(c, rp)
                assert torch.equal(a, c), f"return_halo F={F} step={step}"
        peer.close()
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # pragma: no cover - reported to the parent
        errors.put(f"rank {rank}: {exc!r}")
        raise


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("copy", ["kernel", "engine"])
def test_peer_exchange_matches_nccl_p2p(cuda, copy):
    ctx = mp.get_context("spawn")
    errors = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, errors, copy)) for r in range(2)]
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
