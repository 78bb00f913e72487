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


def time_launches(fn: Callable[[], object], steps: int, warmup: int, device) -> float:
    """Average device time (ms) of one ``fn()``: ``steps`` calls captured in one CUDA graph and replayed between
    two CUDA events on the current stream, after ``warmup`` eager calls and one untimed replay, so host
    overhead does not add to short launches."""
    device = torch.device(device)
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, capture_error_mode="thread_local"):
        for _ in range(steps):
            fn()
    graph.replay()
    stream = torch.cuda.current_stream(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    e0.record(stream)
    graph.replay()
    e1.record(stream)
    torch.cuda.synchronize(device)
    del graph
    return e0.elapsed_time(e1) / steps

