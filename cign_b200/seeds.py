"""Dropout seed streams of the native ops.

Eager calls draw one seed per dropout call from two host counters, exactly
as the reference modules do (collapsed_gat.py:201-211: GAT calls;
fused_block_ops.py:46-50: dropout-LayerNorm / gamma-residual calls):

    GAT call c:         (base + 0x9E3779B97F4A7C15 * (c + 1)) mod 2^63
    block call c, tag:  (base + 0x9E3779B97F4A7C15 * (c + 1) + 0xD2B74407B1CE6E93 * tag) mod 2^63

with base = torch.initial_seed() mod 2^63; calls with p == 0 get seed 0 and
do not advance the counter.

For a training step captured in a CUDA graph, a :class:`DeviceSeedTable`
keeps both counters in device memory.  While a table is active
(``with table.recording():``), each dropout call gets a slot of the table (a
one-element int64 CUDA tensor the kernel reads when it runs) instead of a
value, and ``table.advance()`` -- called once per step, captured with it --
fills the slots of the next step from the device counters and advances
them.  A replayed step therefore draws the same seeds as the same step run
eagerly with the host counters at the same values.
"""
from __future__ import annotations

import contextlib
from typing import List, Optional, Tuple

import torch

from . import _lib

_MASK63 = (1 << 63) - 1
_GOLDEN = 0x9E3779B97F4A7C15
_TAG_MUL = 0xD2B74407B1CE6E93
GAT, BLOCK = 0, 1


class _Counter:
    def __init__(self):
        self.value = 0

    def take(self) -> int:
        v = self.value
        self.value += 1
        return v


_COUNTERS = (_Counter(), _Counter())  # GAT calls, block-op calls
_ACTIVE: Optional["DeviceSeedTable"] = None


def _base() -> int:
    return int(torch.initial_seed()) & _MASK63


def host_seed(kind: int, call: int, tag: int = 0) -> int:
    s = _base() + _GOLDEN * (call + 1)
    if kind == BLOCK:
        s += _TAG_MUL * int(tag)
    return s & _MASK63


def next_seed(kind: int, p: float, tag: int = 0):
    """Seed of the next dropout call of stream `kind` (an int, or a device
    slot while a DeviceSeedTable records)."""
    if float(p) <= 0.0:
        return 0
    if _ACTIVE is not None:
        return _ACTIVE._slot(kind, tag)
    return host_seed(kind, _COUNTERS[kind].take(), tag)


class _CounterIter:
    """Iterator view of one host counter (next() takes a call id)."""

    def __init__(self, kind: int):
        self.kind = kind

    def __iter__(self):
        return self

    def __next__(self) -> int:
        return _COUNTERS[self.kind].take()


def counter_iter(kind: int) -> _CounterIter:
    return _CounterIter(kind)


def host_counters() -> Tuple[int, int]:
    return _COUNTERS[GAT].value, _COUNTERS[BLOCK].value


def set_host_counters(gat: int, block: int) -> None:
    _COUNTERS[GAT].value = int(gat)
    _COUNTERS[BLOCK].value = int(block)


class DeviceSeedTable:
    """Per-step dropout seeds computed on the device (see module docstring)."""

    def __init__(self, device, capacity: int = 256):
        self.device = torch.device(device)
        self.capacity = int(capacity)
        self.values = torch.zeros(self.capacity, dtype=torch.int64, device=self.device)
        self.layout = torch.zeros(3 * self.capacity, dtype=torch.int32, device=self.device)
        self.counters = torch.tensor(list(host_counters()), dtype=torch.int64, device=self.device)
        self.slots: List[Tuple[int, int, int]] = []
        self._per_kind = [0, 0]
        self._uploaded = False

    def _slot(self, kind: int, tag: int) -> torch.Tensor:
        i = len(self.slots)
        if i >= self.capacity:
            raise RuntimeError("DeviceSeedTable capacity exceeded")
        self.slots.append((kind, int(tag), self._per_kind[kind]))
        self._per_kind[kind] += 1
        return self.values[i:i + 1]

    @contextlib.contextmanager
    def recording(self):
        """Dropout calls inside the block take device slots (in call order)."""
        global _ACTIVE
        if _ACTIVE is not None:
            raise RuntimeError("a DeviceSeedTable is already recording")
        self.slots, self._per_kind = [], [0, 0]
        _ACTIVE = self
        try:
            yield self
        finally:
            _ACTIVE = None

    def upload_layout(self) -> None:
        """Copy the recorded slot layout to the device.  Must run outside a
        capture; a captured advance() reads the layout when it is replayed."""
        flat = [v for slot in self.slots for v in slot]
        if flat:
            self.layout[:len(flat)].copy_(torch.tensor(flat, dtype=torch.int32))
        self._uploaded = True

    def advance(self) -> None:
        """Enqueue: fill every slot with the seed of the next step, then
        advance the device counters by the step's call counts."""
        if not self._uploaded and not torch.cuda.is_current_stream_capturing():
            self.upload_layout()
        lib = _lib.load_library()
        with _lib.DeviceGuard(self.device):
            rc = lib.cign_seed_table_step(_base(), len(self.slots), _lib.ptr(self.layout),
                                          _lib.ptr(self.counters), self._per_kind[GAT],
                                          self._per_kind[BLOCK], _lib.ptr(self.values),
                                          _lib.stream_on(self.device))
        _lib.check(rc, "cign_seed_table_step")

    def sync_host_counters(self, prefetched: bool = True) -> None:
        """Continue the eager streams after the steps that used this table.
        With `prefetched`, the table already holds the seeds of one more
        (not yet run) step, whose calls are not counted."""
        g, b = (int(v) for v in self.counters.tolist())
        if prefetched:
            g -= self._per_kind[GAT]
            b -= self._per_kind[BLOCK]
        set_host_counters(g, b)
