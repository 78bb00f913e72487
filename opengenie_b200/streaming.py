"""Host-resident inputs through the block with copies overlapped with compute.

A serving loop that receives latents on the host and must return results to the host runs, for every
step, a host->device copy of the input, the block, and a device->host copy of the result.  Issued back to
back they serialise (two PCIe transfers of 75.5 MB each at L=9216 around a ~1.8 ms block).  Here the
three run on their own CUDA streams with `depth` device buffers, so step i+1's input crosses PCIe while
step i computes and step i-1's result comes back (PCIe is full duplex): the steady-state rate is set by
the slowest of the three, not by their sum.
"""

from __future__ import annotations

from typing import Callable, Sequence

import torch


class HostPipeline:
    def __init__(self, fn: Callable[[torch.Tensor, torch.Tensor], torch.Tensor], shape, dtype, device,
                 depth: int = 2, graphs: bool = False):
        """``fn(x_dev, out_dev)`` runs one step on the current stream, writing ``out_dev``.  With
        ``graphs``, the step on each of the ``depth`` buffer pairs is captured once as a CUDA graph
        (after one eager call, which initialises whatever ``fn`` sets up lazily) and replayed."""
        self.fn = fn
        self.device = torch.device(device)
        self.depth = depth
        self.h2d = torch.cuda.Stream(self.device)
        self.d2h = torch.cuda.Stream(self.device)
        self.comp = torch.cuda.Stream(self.device)
        self.x = [torch.empty(shape, dtype=dtype, device=self.device) for _ in range(depth)]
        self.y = [torch.empty(shape, dtype=dtype, device=self.device) for _ in range(depth)]
        self.in_ready = [torch.cuda.Event() for _ in range(depth)]
        self.computed = [torch.cuda.Event() for _ in range(depth)]
        self.out_done = [torch.cuda.Event() for _ in range(depth)]
        self._used = [False] * depth
        self.graphs = None
        if graphs:
            from .graphs import StepGraph

            with torch.cuda.stream(self.comp):
                for b in range(depth):
                    self.x[b].zero_()
                    fn(self.x[b], self.y[b])
            self.graphs = [StepGraph(lambda b=b: fn(self.x[b], self.y[b]), self.device) for b in range(depth)]

    def run(self, inputs: Sequence[torch.Tensor], outputs: Sequence[torch.Tensor]) -> None:
        """Processes pinned host ``inputs[i]`` into pinned host ``outputs[i]``; asynchronous (returns
        once everything is enqueued; the d2h stream's last event marks completion)."""
        for i, (xin, xout) in enumerate(zip(inputs, outputs)):
            b = i % self.depth
            with torch.cuda.stream(self.h2d):
                if self._used[b]:
                    self.h2d.wait_event(self.computed[b])  # x[b] is free once step i-depth computed
                self.x[b].copy_(xin, non_blocking=True)
                self.in_ready[b].record(self.h2d)
            with torch.cuda.stream(self.comp):
                self.comp.wait_event(self.in_ready[b])
                if self._used[b]:
                    self.comp.wait_event(self.out_done[b])  # y[b] is free once step i-depth was copied out
                if self.graphs is not None:
                    self.graphs[b].replay()
                else:
                    self.fn(self.x[b], self.y[b])
                self.computed[b].record(self.comp)
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(self.computed[b])
                xout.copy_(self.y[b], non_blocking=True)
                self.out_done[b].record(self.d2h)
            self._used[b] = True

    def start_after(self, event: torch.cuda.Event) -> None:
        """Makes the pipeline's streams wait for ``event`` before anything enqueued later."""
        for s in (self.h2d, self.comp, self.d2h):
            s.wait_event(event)

    def wait_streams(self, stream: torch.cuda.Stream) -> None:
        """Makes ``stream`` wait for everything the pipeline enqueued."""
        for s in (self.h2d, self.comp, self.d2h):
            ev = torch.cuda.Event()
            ev.record(s)
            stream.wait_event(ev)
