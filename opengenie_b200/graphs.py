"""A block step captured once as a CUDA graph and replayed.

The block is 5 kernel launches on one GPU (7 with the NVLink exchange's two barriers).  At 8 GPUs a
step is a few hundred microseconds of device work, so issuing the launches from Python each step
makes the host the bottleneck; a graph replay is one launch call.  Every launch in the step takes the
same arguments on every call (buffers are preallocated, the exchange's barrier count lives in device
memory), which is what capture requires.  Capture uses thread-local mode, so other threads may keep
using CUDA while it runs.
"""

from __future__ import annotations

from typing import Callable

import torch


class StepGraph:
    def __init__(self, fn: Callable[[], object], device):
        """Captures ``fn()`` (which must only enqueue work on the current stream and allocate nothing
        that outlives the step) as a graph; ``replay()`` runs it on the caller's current stream."""
        self.device = torch.device(device)
        self.graph = torch.cuda.CUDAGraph()
        torch.cuda.synchronize(self.device)
        with torch.cuda.graph(self.graph, capture_error_mode="thread_local"):
            fn()
        torch.cuda.synchronize(self.device)

    def replay(self) -> None:
        self.graph.replay()
