"""Row-partitioned CIGN over several GPUs (one process per GPU).

Partition (the multi-GPU plan of the reference's hot path: contiguous row
ranges, halo rows exchanged once per hop).  Rank r owns the destination rows
[bounds[r], bounds[r+1]) of every node tensor; the ranges are balanced by
rows + non-zeros of the operator.  The rank's row block of P (and of the GAT
graph, which has the same sparsity pattern as A + I) references columns
outside its range: those "halo" rows are numbered after the rank's own rows,
sorted by global id (so grouped by owner rank), giving the "extended" index
space [own rows | halo rows].

HaloExchange.gather(x_own) -> x_ext fills the halo rows from their owners
(batched NCCL point-to-point sends/receives; gloo on CPU for tests); its
autograd backward sends the halo rows' gradients back to their owners,
which add them to their own rows in a fixed order (peer by peer, unique
indices per peer), so the sum order is deterministic.

On top of it:
  * DistMultiHop: per hop, the SpMM of the rank's row block split by column
    owner -- own columns (square plan) and halo columns (rectangular plan,
    transposes for the backward) -- with the halo rows of the current state
    pushed by their owners while the own-column part runs;
  * DistGatGraph: the aggregate-first collapsed GAT on a rectangular plan
    (destination rows = own rows, source columns = extended rows).
Every other op of the CIGN block is row-local.  Parameter gradients are
summed over ranks with one all-reduce (allreduce_gradients).
"""
from __future__ import annotations

from typing import Dict, List, Optional, Sequence

import torch
import torch.distributed as dist

from .plans import SpmmPlan


# Cost of an own row relative to a non-zero in the partition balance.  On the
# 2.45M-node RMAT graph at 8 ranks (two partitions measured), a rank's busy
# time per step fitted 159 ns per own row (the row-wise ops, the GEMMs and
# the per-row fixed cost of the gathers) + 3.2 ns per non-zero + 34 ms, so a
# row weighs 50 non-zeros.
ROW_WEIGHT = 50


def partition_rows(crow: torch.Tensor, world: int, row_weight: int = 1) -> List[int]:
    """Contiguous row ranges [b[r], b[r+1]) balancing row_weight * rows +
    non-zeros."""
    crow = crow.to(torch.int64).cpu()
    n = crow.numel() - 1
    nnz = int(crow[-1])
    # work before each row start
    work = crow + int(row_weight) * torch.arange(n + 1, dtype=torch.int64)
    total = int(row_weight) * n + nnz
    bounds = [0]
    for r in range(1, world):
        t = (r * total) // world
        b = int(torch.searchsorted(work, torch.tensor(t), right=False))
        bounds.append(max(bounds[-1], min(b, n)))
    bounds.append(n)
    return bounds


class HaloPlan:
    """Index bookkeeping of one rank (computed identically on every rank from
    the global CSR; no communication)."""

    def __init__(self, crow: torch.Tensor, col: torch.Tensor, bounds: Sequence[int], rank: int):
        crow = crow.to(torch.int64).cpu()
        col = col.to(torch.int64).cpu()
        self.bounds = list(bounds)
        self.rank = rank
        self.world = len(bounds) - 1
        r0, r1 = self.bounds[rank], self.bounds[rank + 1]
        self.r0, self.r1 = r0, r1
        self.n_own = r1 - r0
        block = col[int(crow[r0]):int(crow[r1])]
        outside = block[(block < r0) | (block >= r1)]
        self.halo = torch.unique(outside)  # sorted global ids
        self.n_halo = int(self.halo.numel())
        b = torch.tensor(self.bounds, dtype=torch.int64)
        owner = torch.searchsorted(b, self.halo, right=True) - 1
        self.recv_counts = [int((owner == p).sum()) for p in range(self.world)]
        self.send_idx: List[torch.Tensor] = []
        self.send_counts: List[int] = []
        for p in range(self.world):
            if p == rank:
                self.send_idx.append(torch.zeros(0, dtype=torch.int64))
                self.send_counts.append(0)
                continue
            p0, p1 = self.bounds[p], self.bounds[p + 1]
            pc = col[int(crow[p0]):int(crow[p1])]
            need = torch.unique(pc[(pc >= r0) & (pc < r1)]) - r0
            self.send_idx.append(need)
            self.send_counts.append(int(need.numel()))

    def to_ext(self, cols: torch.Tensor) -> torch.Tensor:
        """Global column ids -> extended ids ([own rows | halo rows])."""
        cols = cols.to(torch.int64).cpu()
        own = (cols >= self.r0) & (cols < self.r1)
        ext = torch.empty_like(cols)
        ext[own] = cols[own] - self.r0
        pos = torch.searchsorted(self.halo, cols[~own])
        if pos.numel() and (pos.max() >= self.n_halo or not torch.equal(self.halo[pos], cols[~own])):
            raise ValueError("column outside this rank's halo")
        ext[~own] = self.n_own + pos
        return ext


class TorchP2P:
    """Point-to-point transport over torch.distributed (NCCL between GPUs,
    gloo on CPU): one batched group of sends and receives per exchange."""

    def __init__(self, group=None):
        self.group = group

    def exchange(self, sends: Dict[int, torch.Tensor], recvs: Dict[int, torch.Tensor]) -> None:
        ops = []
        for p in sorted(set(sends) | set(recvs)):
            if p in sends:
                ops.append(dist.P2POp(dist.isend, sends[p], p, self.group))
            if p in recvs:
                ops.append(dist.P2POp(dist.irecv, recvs[p], p, self.group))
        if ops:
            for req in dist.batch_isend_irecv(ops):
                req.wait()


class StagedGlooP2P:
    """Point-to-point transport staged through host memory over a gloo
    group: for ranks that cannot use NCCL between them (e.g. several
    processes sharing one GPU in tests).  Slower than TorchP2P."""

    def __init__(self, group=None):
        self.group = group

    def exchange(self, sends: Dict[int, torch.Tensor], recvs: Dict[int, torch.Tensor]) -> None:
        host_recv = {p: torch.empty(t.shape, dtype=t.dtype) for p, t in recvs.items()}
        ops = []
        for p in sorted(set(sends) | set(recvs)):
            if p in sends:
                ops.append(dist.P2POp(dist.isend, sends[p].detach().cpu(), p, self.group))
            if p in recvs:
                ops.append(dist.P2POp(dist.irecv, host_recv[p], p, self.group))
        if ops:
            for req in dist.batch_isend_irecv(ops):
                req.wait()
        for p, t in recvs.items():
            t.copy_(host_recv[p])


class LoopbackTransport:
    """In-process transport between ranks run as threads of one process (all
    on one device and stream): rank r's send to p is a copy queued for p.
    For tests of the partitioned path on a single GPU."""

    def __init__(self, world: int):
        import queue
        self.world = world
        self.boxes = {(a, b): queue.Queue() for a in range(world) for b in range(world)}

    def endpoint(self, rank: int) -> "LoopbackTransport._Endpoint":
        return LoopbackTransport._Endpoint(self, rank)

    class _Endpoint:
        def __init__(self, hub, rank):
            self.hub, self.rank = hub, rank

        def exchange(self, sends, recvs):
            for p, t in sends.items():
                self.hub.boxes[(self.rank, p)].put(t.clone())
            for p, t in recvs.items():
                t.copy_(self.hub.boxes[(p, self.rank)].get(timeout=120))


class HaloExchange:
    def __init__(self, plan: HaloPlan, device, transport=None):
        self.plan = plan
        self.device = torch.device(device)
        self.transport = transport if transport is not None else TorchP2P()
        self.n_own, self.n_halo = plan.n_own, plan.n_halo
        self.send_idx = [t.to(self.device) for t in plan.send_idx]
        self.send_all = (torch.cat(self.send_idx) if plan.world > 1
                         else torch.zeros(0, dtype=torch.int64, device=self.device))
        self.send_off = _offsets(plan.send_counts)
        self.recv_off = _offsets(plan.recv_counts)

    def _exchange(self, sends: Dict[int, torch.Tensor], recvs: Dict[int, torch.Tensor]) -> None:
        self.transport.exchange(sends, recvs)

    def begin_step(self) -> None:
        """Called at the start of every training step (buffer bookkeeping of
        exchanges that keep per-step buffers; nothing to do here)."""

    def gather(self, x_own: torch.Tensor) -> torch.Tensor:
        """x_ext [n_own + n_halo, F]: own rows, then the halo rows from their owners."""
        F = x_own.size(1)
        x_ext = torch.empty((self.n_own + self.n_halo, F), dtype=x_own.dtype, device=x_own.device)
        x_ext[:self.n_own].copy_(x_own)
        send = x_own.index_select(0, self.send_all) if self.send_all.numel() else None
        sends, recvs = {}, {}
        for p in range(self.plan.world):
            if self.plan.send_counts[p]:
                sends[p] = send[self.send_off[p]:self.send_off[p] + self.plan.send_counts[p]]
            if self.plan.recv_counts[p]:
                a = self.n_own + self.recv_off[p]
                recvs[p] = x_ext[a:a + self.plan.recv_counts[p]]
        self._exchange(sends, recvs)
        return x_ext

    def gather_halo(self, x_own: torch.Tensor):
        """Start filling the halo rows only: returns (halo [n_halo, F], event).
        The caller's stream must wait for `event` (None: already complete)
        before reading halo."""
        F = x_own.size(1)
        halo = torch.empty((self.n_halo, F), dtype=x_own.dtype, device=x_own.device)
        send = x_own.index_select(0, self.send_all) if self.send_all.numel() else None
        sends, recvs = {}, {}
        for p in range(self.plan.world):
            if self.plan.send_counts[p]:
                sends[p] = send[self.send_off[p]:self.send_off[p] + self.plan.send_counts[p]]
            if self.plan.recv_counts[p]:
                recvs[p] = halo[self.recv_off[p]:self.recv_off[p] + self.plan.recv_counts[p]]
        self._exchange(sends, recvs)
        return halo, None

    def return_halo(self, g_halo: torch.Tensor):
        """Start sending the halo rows' gradients [n_halo, F] back to their
        owners: returns (recv [sum(send_counts), F], event) for add_returned."""
        g_halo = g_halo.contiguous()
        F = g_halo.size(1)
        recv = torch.empty((int(self.send_all.numel()), F), dtype=g_halo.dtype,
                           device=g_halo.device)
        sends, recvs = {}, {}
        for p in range(self.plan.world):
            if self.plan.recv_counts[p]:
                sends[p] = g_halo[self.recv_off[p]:self.recv_off[p] + self.plan.recv_counts[p]]
            if self.plan.send_counts[p]:
                recvs[p] = recv[self.send_off[p]:self.send_off[p] + self.plan.send_counts[p]]
        self._exchange(sends, recvs)
        return recv, None

    def add_returned(self, g_own: torch.Tensor, recv: torch.Tensor) -> None:
        """g_own += the gradients the peers returned (peer by peer, fixed order)."""
        for p in range(self.plan.world):
            c = self.plan.send_counts[p]
            if c:
                g_own.index_add_(0, self.send_idx[p], recv[self.send_off[p]:self.send_off[p] + c])

    def scatter_add(self, g_ext: torch.Tensor) -> torch.Tensor:
        """Backward of gather: own rows' gradient plus the gradients other
        ranks computed for them (added peer by peer)."""
        g_ext = g_ext.contiguous()
        F = g_ext.size(1)
        g_own = g_ext[:self.n_own].clone()
        recv = torch.empty((int(self.send_all.numel()), F), dtype=g_ext.dtype, device=g_ext.device)
        sends, recvs = {}, {}
        for p in range(self.plan.world):
            if self.plan.recv_counts[p]:
                a = self.n_own + self.recv_off[p]
                sends[p] = g_ext[a:a + self.plan.recv_counts[p]]
            if self.plan.send_counts[p]:
                recvs[p] = recv[self.send_off[p]:self.send_off[p] + self.plan.send_counts[p]]
        self._exchange(sends, recvs)
        for p in range(self.plan.world):
            if self.plan.send_counts[p]:
                g_own.index_add_(0, self.send_idx[p], recvs[p])
        return g_own


class _DeviceArray:
    """Zero-copy torch view of a raw device allocation (CUDA array interface)."""

    def __init__(self, ptr: int, shape, device: torch.device):
        self.__cuda_array_interface__ = {"data": (int(ptr), False), "shape": tuple(shape),
                                         "typestr": "<f4", "strides": None, "version": 3}
        self.device = device


class PeerHaloExchange(HaloExchange):
    """Halo exchange over NVLink peer memory instead of NCCL point-to-point.

    Every exchange of a step gets its own buffers (allocated on first use with
    cudaMalloc, shared with the peers through CUDA IPC): for a gather, the
    extended tensor [own rows | halo rows] into whose halo part the owners
    store their rows with cign_halo_push; for a scatter_add, the buffer into
    which the peers store the gradients of the rows this rank sent them.
    One collective after each push orders the stores before any rank reads.
    Buffers are reused by the same exchange of the next step; the
    gradient all-reduce that ends every step orders those writes after the
    previous step's reads.  Call begin_step() at the start of every step.
    """

    def __init__(self, plan: HaloPlan, device, group=None, copy: str = "kernel"):
        super().__init__(plan, device, TorchP2P(group))
        from . import _lib
        if copy not in ("kernel", "engine"):
            raise ValueError("copy must be 'kernel' (SM stores) or 'engine' (copy engines)")
        self.lib = _lib.load_library()
        self._lib = _lib
        self.group = group
        self.copy = copy
        w = plan.world
        # every rank's counts, so each rank can address its slots on the peers
        mine = torch.tensor([plan.n_own] + plan.recv_counts + plan.send_counts,
                            dtype=torch.int64, device=self.device)
        allc = [torch.empty_like(mine) for _ in range(w)]
        dist.all_gather(allc, mine, group=group)
        allc = [t.cpu().tolist() for t in allc]
        self.n_own_of = [a[0] for a in allc]
        self.recv_off_of = [_offsets(a[1:1 + w]) for a in allc]
        self.send_off_of = [_offsets(a[1 + w:1 + 2 * w]) for a in allc]
        self.send_begin = torch.tensor(_offsets(plan.send_counts) + [sum(plan.send_counts)],
                                       dtype=torch.int64, device=self.device)
        self.recv_begin = torch.tensor(_offsets(plan.recv_counts) + [sum(plan.recv_counts)],
                                       dtype=torch.int64, device=self.device)
        first = (plan.rank + 1) % w
        self._order = {  # kernel pushes: rows interleaved over the peers
            "send": interleaved_order(plan.send_counts, first).to(self.device),
            "recv": interleaved_order(plan.recv_counts, first).to(self.device)}
        self._first_peer = first  # copy-engine pushes: peers in turn from rank + 1
        self._begin_host = {  # the same offsets as host arrays (copy-engine pushes)
            "send": (_lib.ctypes.c_int64 * (w + 1))(*(_offsets(plan.send_counts)
                                                       + [sum(plan.send_counts)])),
            "recv": (_lib.ctypes.c_int64 * (w + 1))(*(_offsets(plan.recv_counts)
                                                       + [sum(plan.recv_counts)]))}
        self._flag = torch.zeros(1, dtype=torch.float32, device=self.device)
        self._slots: List[dict] = []
        self._call = 0
        self._stream = None  # side stream of the asynchronous pushes
        # list to collect (start, push done, barrier done, bytes sent) of every
        # push and its ordering collective, or None (set by benchmarks; not
        # used under graph capture)
        self.timer = None

    def begin_step(self, order_with_previous_step: bool = False) -> None:
        """Start a step: the exchanges of this step reuse the previous step's
        buffers, in the same order.  A peer's push of this step overwrites a
        buffer this rank read in the previous step, so some collective must
        separate the two steps on every rank.  A training step has one (the
        gradient all-reduce at its end); a caller without one -- e.g. forward
        passes only, for evaluation -- passes order_with_previous_step=True,
        which adds a one-element all-reduce on the current stream here.  Every
        rank must pass the same value."""
        self._call = 0
        if order_with_previous_step:
            dist.all_reduce(self._flag, group=self.group)

    def _alloc_shared(self, rows: int, F: int):
        """A [rows, F] fp32 buffer of this rank and the base pointers of every
        rank's buffer of the same slot (all ranks allocate together)."""
        nbytes = max(int(rows) * int(F) * 4, 16)
        ptr = self._lib.c_void_p()
        rc = self.lib.cign_device_alloc(nbytes, self._lib.ctypes.byref(ptr))
        if rc != 0:  # memory cached by torch's allocator: release it and retry once
            torch.cuda.synchronize(self.device)
            torch.cuda.empty_cache()
            rc = self.lib.cign_device_alloc(nbytes, self._lib.ctypes.byref(ptr))
        # every rank learns whether all allocations succeeded before any of
        # them waits in the handle exchange
        ok = torch.tensor([1.0 if rc == 0 else 0.0], device=self.device)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=self.group)
        if float(ok.item()) < 1.0:
            if rc == 0:
                self.lib.cign_device_free(ptr)
            raise RuntimeError(f"peer halo buffer of {nbytes} bytes: cudaMalloc failed on "
                               f"{'this' if rc != 0 else 'another'} rank (out of device memory)")
        handle = (self._lib.ctypes.c_ubyte * 64)()
        self._lib.check(self.lib.cign_ipc_handle(ptr, handle), "cign_ipc_handle")
        mine = torch.tensor(list(handle), dtype=torch.uint8, device=self.device)
        allh = [torch.empty_like(mine) for _ in range(self.plan.world)]
        dist.all_gather(allh, mine, group=self.group)
        bases = []
        for r, h in enumerate(allh):
            if r == self.plan.rank:
                bases.append(ptr.value)
                continue
            hb = (self._lib.ctypes.c_ubyte * 64)(*h.cpu().tolist())
            q = self._lib.c_void_p()
            self._lib.check(self.lib.cign_ipc_open(hb, self._lib.ctypes.byref(q)), "cign_ipc_open")
            bases.append(q.value)
        view = torch.as_tensor(_DeviceArray(ptr.value, (rows, F), self.device), device=self.device)
        return ptr, view, bases

    def _slot(self, kind: str, F: int) -> dict:
        i = self._call
        self._call += 1
        if i < len(self._slots):
            slot = self._slots[i]
            if slot["kind"] != kind or slot["F"] != F:
                raise RuntimeError("exchange sequence changed between steps")
            return slot
        me, w = self.plan.rank, self.plan.world
        if kind == "gather":
            ptr, view, bases = self._alloc_shared(self.n_own + self.n_halo, F)
            dst = [bases[p] + (self.n_own_of[p] + self.recv_off_of[p][me]) * F * 4
                   for p in range(w)]
        elif kind == "halo":  # the halo rows only
            ptr, view, bases = self._alloc_shared(self.n_halo, F)
            dst = [bases[p] + self.recv_off_of[p][me] * F * 4 for p in range(w)]
        else:  # scatter: peers store gradients of the rows this rank sent them
            ptr, view, bases = self._alloc_shared(int(self.send_all.numel()), F)
            dst = [bases[p] + self.send_off_of[p][me] * F * 4 for p in range(w)]
        slot = {"kind": kind, "F": F, "ptr": ptr, "view": view, "bases": bases,
                "dst": torch.tensor(dst, dtype=torch.int64, device=self.device),
                "dst_host": (self._lib.ctypes.c_void_p * w)(*dst),
                # copy engines: the gathered send rows, contiguous per peer
                "staging": (torch.empty((int(self.send_all.numel()), F), dtype=torch.float32,
                                        device=self.device)
                            if self.copy == "engine" and kind != "scatter" else None)}
        self._slots.append(slot)
        return slot

    def _push(self, src, F, idx, slot, total):
        stream = torch.cuda.current_stream(self.device)
        if self.timer is not None:
            t0 = torch.cuda.Event(enable_timing=True)
            t0.record(stream)
        gathered = idx is not None  # send rows of x (gather) or halo-row gradients (scatter)
        if self.copy == "engine":
            rc = self.lib.cign_halo_push_copy(
                self.plan.world, self._lib.ptr(src), F, self._lib.ptr(idx) if gathered else None,
                self._begin_host["send" if gathered else "recv"], slot["dst_host"], int(total),
                self._lib.ptr(slot["staging"]) if gathered else None, self._first_peer,
                self._lib.stream_of(src))
            self._lib.check(rc, "cign_halo_push_copy")
        else:
            begin = self.send_begin if gathered else self.recv_begin
            order = self._order["send" if gathered else "recv"]
            rc = self.lib.cign_halo_push(self.plan.world, self._lib.ptr(src), F,
                                         self._lib.ptr(idx) if gathered else None,
                                         self._lib.ptr(begin), self._lib.ptr(slot["dst"]),
                                         int(total), self._lib.ptr(order) if order.numel() else None,
                                         self._lib.stream_of(src))
            self._lib.check(rc, "cign_halo_push")
        if self.timer is not None:
            t1 = torch.cuda.Event(enable_timing=True)
            t1.record(stream)
        dist.all_reduce(self._flag, group=self.group)  # all stores done before any read
        if self.timer is not None:
            t2 = torch.cuda.Event(enable_timing=True)
            t2.record(stream)
            self.timer.append((t0, t1, t2, int(total) * int(F) * 4))

    def _side(self):
        if self._stream is None:
            self._stream = torch.cuda.Stream(self.device)
        return self._stream

    def _push_async(self, src, F, idx, slot, total):
        """The push and its ordering collective on the side stream, after the
        current stream's work so far; returns the event that ends them."""
        cur = torch.cuda.current_stream(self.device)
        side = self._side()
        side.wait_stream(cur)
        with torch.cuda.stream(side):
            self._push(src, F, idx, slot, total)
            ev = torch.cuda.Event()
            ev.record(side)
        return ev

    def gather_halo(self, x_own: torch.Tensor):
        x_own = x_own.contiguous()
        F = int(x_own.size(1))
        slot = self._slot("halo", F)
        ev = self._push_async(x_own, F, self.send_all, slot, int(self.send_all.numel()))
        return slot["view"], ev

    def return_halo(self, g_halo: torch.Tensor):
        g_halo = g_halo.contiguous()
        F = int(g_halo.size(1))
        slot = self._slot("scatter", F)
        ev = self._push_async(g_halo, F, None, slot, self.n_halo)
        return slot["view"], ev

    def gather(self, x_own: torch.Tensor) -> torch.Tensor:
        x_own = x_own.contiguous()
        F = int(x_own.size(1))
        slot = self._slot("gather", F)
        x_ext = slot["view"]
        x_ext[:self.n_own].copy_(x_own)
        self._push(x_own, F, self.send_all, slot, int(self.send_all.numel()))
        return x_ext

    def scatter_add(self, g_ext: torch.Tensor) -> torch.Tensor:
        g_ext = g_ext.contiguous()
        F = int(g_ext.size(1))
        slot = self._slot("scatter", F)
        g_own = g_ext[:self.n_own].clone()
        self._push(g_ext[self.n_own:], F, None, slot, self.n_halo)
        recv = slot["view"]
        for p in range(self.plan.world):
            c = self.plan.send_counts[p]
            if c:
                g_own.index_add_(0, self.send_idx[p], recv[self.send_off[p]:self.send_off[p] + c])
        return g_own

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (after the last step)."""
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for slot in self._slots:
            for r, b in enumerate(slot["bases"]):
                if r != self.plan.rank:
                    self.lib.cign_ipc_close(self._lib.c_void_p(b))
        dist.barrier(group=self.group)
        for slot in self._slots:
            self.lib.cign_device_free(slot["ptr"])
        self._slots = []


def interleaved_order(counts: Sequence[int], first: int) -> torch.Tensor:
    """Flat indices of a list made of consecutive per-peer blocks (block p
    holds counts[p] rows), visited round-robin over the peers starting at
    peer `first`: row 0 of every peer, then row 1 of every peer, ...  Pushed
    in this order, every rank's stores spread over all its peers' links at
    once instead of all ranks storing into the same peer first."""
    w = len(counts)
    offs = _offsets(counts)
    keys, flat = [], []
    for p, c in enumerate(counts):
        if c == 0:
            continue
        j = torch.arange(int(c), dtype=torch.int64)
        keys.append(j * w + (p - first) % w)
        flat.append(offs[p] + j)
    if not keys:
        return torch.zeros(0, dtype=torch.int64)
    keys, flat = torch.cat(keys), torch.cat(flat)
    return flat[torch.argsort(keys)]


def _offsets(counts: Sequence[int]) -> List[int]:
    out, acc = [], 0
    for c in counts:
        out.append(acc)
        acc += int(c)
    return out


class _HaloFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x_own, exchange):
        ctx.exchange = exchange
        return exchange.gather(x_own.contiguous())

    @staticmethod
    def backward(ctx, g_ext):
        return ctx.exchange.scatter_add(g_ext), None


def halo_gather(x_own: torch.Tensor, exchange: HaloExchange) -> torch.Tensor:
    return _HaloFn.apply(x_own, exchange)


def _local_block(crow, col, val, plan: HaloPlan):
    """Rows [r0, r1) of a global CSR with extended column ids (edge order kept)."""
    crow = crow.to(torch.int64).cpu()
    a, b = int(crow[plan.r0]), int(crow[plan.r1])
    lcrow = crow[plan.r0:plan.r1 + 1] - a
    lcol = plan.to_ext(col[a:b])
    lval = None if val is None else val[a:b].cpu()
    return lcrow, lcol, lval


def _csr_plan(rows_of_edges, cols, vals, n_rows: int, n_cols: int, dev) -> SpmmPlan:
    """SpmmPlan of the [n_rows, n_cols] operator given as COO edges (row-major
    order kept), with its transpose for the backward."""
    counts = torch.bincount(rows_of_edges, minlength=n_rows)
    crow = torch.zeros(n_rows + 1, dtype=torch.int64)
    crow[1:] = torch.cumsum(counts, 0)
    t = torch.sparse_coo_tensor(torch.stack([cols, rows_of_edges]), vals,
                                (n_cols, n_rows)).coalesce().to_sparse_csr()
    return SpmmPlan(crow.to(dev), cols.to(dev), vals.to(dev), t.crow_indices().to(dev),
                    t.col_indices().to(dev), t.values().to(dev), cols=n_cols)


class _DistHopFn(torch.autograd.Function):
    """One hop y = P_r x over the rank's row block as an autograd node
    (DistMultiHop.hop_forward / hop_backward)."""

    @staticmethod
    def forward(ctx, x_own, hop: "DistMultiHop"):
        ctx.hop = hop
        return hop.hop_forward(x_own)

    @staticmethod
    def backward(ctx, g):
        return ctx.hop.hop_backward(g), None


class DistMultiHop:
    """k-hop propagation P^p x over the row-partitioned operator; each hop
    overlaps the halo exchange with the own-column part of the SpMM.

    Besides the autograd form (powers), it offers the raw forward/backward
    pair of a native SpmmPlan (forward(x, K), backward(grads, F)), so the
    block's fused propagate + hop gate + pack node runs on it unchanged."""

    is_row_partitioned = True

    def __init__(self, csr_global: torch.Tensor, plan: HaloPlan, exchange: HaloExchange):
        crow = csr_global.crow_indices().cpu()
        col = csr_global.col_indices().cpu()
        val = csr_global.values().cpu()
        lcrow, lcol, lval = _local_block(crow, col, val, plan)
        n_own = plan.n_own
        rows = torch.repeat_interleave(torch.arange(n_own), lcrow[1:] - lcrow[:-1])
        dev = exchange.device
        own = lcol < n_own
        self.own = _csr_plan(rows[own], lcol[own], lval[own], n_own, n_own, dev)
        hal = ~own
        self.halo = (_csr_plan(rows[hal], lcol[hal] - n_own, lval[hal], n_own, plan.n_halo, dev)
                     if plan.n_halo else None)
        self.exchange = exchange
        self.nnz_local = int(lcol.numel())

    def hop_forward(self, x_own: torch.Tensor) -> torch.Tensor:
        """y = P_own x_own + P_halo halo(x): the owners push this rank's halo
        rows on a side stream while P_own x_own is computed."""
        x_own = x_own.contiguous()
        halo, ev = self.exchange.gather_halo(x_own)
        y = self.own.spmm(x_own)
        if ev is not None:
            torch.cuda.current_stream(x_own.device).wait_event(ev)
        if self.halo is None:
            return y
        return self.halo.spmm(halo, addend=y)

    def hop_backward(self, g: torch.Tensor,
                     addend: Optional[torch.Tensor] = None) -> torch.Tensor:
        """P_r^T g (+ addend): P_halo^T g goes back to the owners on the side
        stream while P_own^T g (+ addend) is computed; the rows the peers
        returned are added in a fixed peer order."""
        g = g.contiguous()
        # a rank without halo columns returns nothing but still takes the
        # exchange's steps (its collective) like every other rank
        g_halo = (g.new_zeros((0, g.size(1))) if self.halo is None
                  else self.halo.spmm(g, transpose=True))
        recv, ev = self.exchange.return_halo(g_halo)
        g_own = self.own.spmm(g, transpose=True, addend=addend)
        if ev is not None:
            torch.cuda.current_stream(g.device).wait_event(ev)
        self.exchange.add_returned(g_own, recv)
        return g_own

    def powers(self, x_own: torch.Tensor, powers: Sequence[int]) -> Dict[int, torch.Tensor]:
        wanted = sorted(set(int(p) for p in powers))
        out: Dict[int, torch.Tensor] = {}
        if 0 in wanted:
            out[0] = x_own
        cur = x_own
        for p in range(1, wanted[-1] + 1):
            cur = _DistHopFn.apply(cur, self)
            if p in wanted:
                out[p] = cur
        return out

    def forward(self, x_own: torch.Tensor, max_power: int) -> List[torch.Tensor]:
        """[P^1 x, ..., P^max_power x] over the rank's rows (no autograd)."""
        ys, cur = [], x_own
        for _ in range(int(max_power)):
            cur = self.hop_forward(cur)
            ys.append(cur)
        return ys

    def backward(self, grads: Sequence[Optional[torch.Tensor]], F: int) -> torch.Tensor:
        """grads[p-1] = dL/d(P^p x) or None (the last one given); returns
        dL/dx = sum_p (P^T)^p grads[p-1], accumulated from the highest hop down
        with each lower hop's gradient added inside the SpMM."""
        if grads[-1] is None:
            raise ValueError("the highest hop's gradient must be given")
        acc = grads[-1]
        for p in range(len(grads) - 1, 0, -1):
            acc = self.hop_backward(acc, grads[p - 1])
        return self.hop_backward(acc)


class DistGatGraph:
    """The rank's block of the GAT graph ((rowptr, col), (row, colptr), perm)
    over extended columns, with the halo exchange that fills them."""

    def __init__(self, rowptr_g: torch.Tensor, col_g: torch.Tensor, plan: HaloPlan,
                 exchange: HaloExchange):
        lcrow, lcol, _ = _local_block(rowptr_g, col_g, None, plan)
        n_own, n_ext = plan.n_own, plan.n_own + plan.n_halo
        nnz = int(lcol.numel())
        rows = torch.repeat_interleave(torch.arange(n_own), lcrow[1:] - lcrow[:-1])
        # CSC over extended columns; perm[csc position] = local CSR edge id
        order = torch.argsort(lcol * max(n_own, 1) + rows, stable=True)
        row_csc = rows[order]
        counts = torch.bincount(lcol, minlength=n_ext)
        colptr = torch.zeros(n_ext + 1, dtype=torch.int64)
        colptr[1:] = torch.cumsum(counts, 0)
        dev = exchange.device
        i32 = lambda t: t.to(torch.int32).to(dev)  # noqa: E731
        self.csr = (i32(lcrow), i32(lcol))
        self.csc = (i32(row_csc), i32(colptr))
        self.perm = i32(order)
        self.exchange = exchange
        self.n_own, self.n_ext, self.nnz = n_own, n_ext, nnz

    def halo(self, x_own: torch.Tensor) -> torch.Tensor:
        return halo_gather(x_own, self.exchange)


def partition_graph(csr_global: torch.Tensor, gat_rowptr: torch.Tensor, gat_col: torch.Tensor,
                    world: int, rank: int, device, transport=None, row_weight: int = ROW_WEIGHT):
    """Everything one rank needs: (bounds, HaloPlan, HaloExchange, DistMultiHop,
    DistGatGraph).  csr_global: P as a sparse CSR tensor; gat_rowptr/gat_col:
    the destination-major CSR of the GAT graph (same sparsity pattern).
    transport: None (NCCL point-to-point), "peer" (NVLink peer-memory stores
    by a kernel, PeerHaloExchange), "peer-copy" (the same buffers filled by
    the copy engines), or a transport object (TorchP2P, StagedGlooP2P, ...).
    row_weight: cost of an own row in units of one non-zero (partition_rows)."""
    bounds = partition_rows(csr_global.crow_indices(), world, row_weight)
    plan = HaloPlan(csr_global.crow_indices(), csr_global.col_indices(), bounds, rank)
    if transport in ("peer", "peer-copy"):
        exchange = PeerHaloExchange(plan, device, copy="engine" if transport == "peer-copy"
                                    else "kernel")
    else:
        exchange = HaloExchange(plan, device, transport)
    op = DistMultiHop(csr_global, plan, exchange)
    gat = DistGatGraph(gat_rowptr, gat_col, plan, exchange)
    return bounds, plan, exchange, op, gat


def allreduce_gradients(params, group=None) -> None:
    """Sum every parameter's gradient over the ranks (one flat all-reduce)."""
    grads = [p.grad for p in params if p.grad is not None]
    if not grads:
        return
    flat = torch.cat([g.reshape(-1) for g in grads])
    dist.all_reduce(flat, group=group)
    off = 0
    for g in grads:
        n = g.numel()
        g.copy_(flat[off:off + n].view_as(g))
        off += n
