"""A whole training step captured in one CUDA graph.

The reference runs every step eagerly from Python (generic_engine/train_cign.py:2103-2148),
which costs several milliseconds of host time per step at cfg2 scale -- more
than the device needs.  :class:`GraphedStep` runs a step function a few
times eagerly (on a side stream, so lazy initialisation happens outside the
capture), captures one step in a CUDA graph and then replays it.

Requirements on ``step_fn``: it runs forward, loss, backward and the
optimizer step on static input tensors (same storage every call), returns
the loss tensor, and never synchronises with the host (no boolean-mask
indexing, no ``.item()``).  Optimizers must be built with
``capturable=True``.  Dropout of the native ops draws its seeds from a
:class:`cign_b200.seeds.DeviceSeedTable` (the same per-call seeds as eager
execution with the same call counters); torch's own dropout uses torch's
graph-safe generator.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch

from . import _lib
from .seeds import DeviceSeedTable


class GraphedStep:
    def __init__(self, step_fn: Callable[[], torch.Tensor], device, warmup: int = 3,
                 before_capture: Optional[Callable[[], None]] = None):
        self.device = torch.device(device)
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(max(1, int(warmup))):
                step_fn()
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)
        if before_capture is not None:
            before_capture()
        self.seeds = DeviceSeedTable(self.device)
        self.graph = torch.cuda.CUDAGraph()
        lib = _lib.load_library()
        launches0 = int(lib.cign_kernel_launches())
        with self.seeds.recording():
            with torch.cuda.graph(self.graph):
                self.loss = step_fn()
                self.seeds.advance()  # seeds of the next replay
        # this library's kernels in one replay (counted as they were captured)
        self.native_launches = int(lib.cign_kernel_launches()) - launches0
        self.seeds.upload_layout()
        self.seeds.advance()  # seeds of the first replay
        torch.cuda.synchronize(self.device)

    def __call__(self) -> torch.Tensor:
        """Replay one step on the current stream; returns the (static) loss tensor."""
        self.graph.replay()
        return self.loss

    def finish(self) -> None:
        """Hand the dropout call counters back to the eager streams."""
        torch.cuda.synchronize(self.device)
        self.seeds.sync_host_counters()
