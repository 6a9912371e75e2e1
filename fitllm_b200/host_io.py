"""Host <-> device batch pipeline: PCIe copies overlapped with the step.

The reference moves every micro-batch's hidden states between pinned host
memory and the device on the compute stream, inside its layer loop
(fitllm/forward.py:480-528, fitllm/backward.py:206-249), so each copy
serialises with the kernels around it.  Here a training loop that takes its
inputs from, and returns its results to, pinned host memory runs its steps
through ``HostBatchPipeline``:

* the host->device copy of batch i+1 runs on its own stream while step i
  computes (``depth`` device buffers per input, reused in turn once the step
  that read them has finished);
* step i's results are copied to their pinned host buffers on a third stream
  once step i's kernels are done, while step i+1 computes;
* at the end the caller's stream waits for the last copy, so an event
  recorded on it after ``run`` covers every copy.

All copies of every step still happen; only their overlap with compute
changes.  Results are bit-identical to issuing the same copies in stream
order (tested).
"""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence

import torch


class HostBatchPipeline:
    """``templates``: one pinned host tensor per step input (shape and dtype
    of every batch's inputs)."""

    def __init__(self, device, templates: Sequence[torch.Tensor], depth: int = 2):
        if depth < 1:
            raise ValueError("HostBatchPipeline: depth must be >= 1")
        self.device = torch.device(device)
        self.depth = depth
        self.h2d = torch.cuda.Stream(device=self.device)
        self.d2h = torch.cuda.Stream(device=self.device)
        self.bufs = [[torch.empty(t.shape, dtype=t.dtype, device=self.device) for t in templates]
                     for _ in range(depth)]
        self.ready = [torch.cuda.Event() for _ in range(depth)]
        self.free: List[Optional[torch.cuda.Event]] = [None] * depth
        self.h2d_bytes = 0
        self.d2h_bytes = 0

    def _upload(self, slot: int, batch: Sequence[torch.Tensor]) -> None:
        if len(batch) != len(self.bufs[slot]):
            raise ValueError("HostBatchPipeline: batch has the wrong number of inputs")
        if self.free[slot] is not None:
            self.h2d.wait_event(self.free[slot])
        with torch.cuda.stream(self.h2d):
            for dst, src in zip(self.bufs[slot], batch):
                if not src.is_pinned():
                    raise ValueError("HostBatchPipeline: host inputs must be pinned")
                dst.copy_(src, non_blocking=True)
                self.h2d_bytes += src.numel() * src.element_size()
            self.ready[slot].record(self.h2d)

    def run(self, step_fn: Callable[[List[torch.Tensor]], Sequence[torch.Tensor]],
            batches: Sequence[Sequence[torch.Tensor]],
            outputs: Sequence[Sequence[torch.Tensor]]) -> None:
        """For each i: ``outs = step_fn(device inputs of batches[i])`` on the
        current stream, then ``outputs[i][j].copy_(outs[j])`` (pinned host).
        ``step_fn`` must return tensors that later steps do not modify."""
        if len(outputs) != len(batches):
            raise ValueError("HostBatchPipeline: one output list per batch")
        if not batches:
            return
        compute = torch.cuda.current_stream(self.device)
        # copies start after everything the caller queued (e.g. a timing event)
        self.h2d.wait_stream(compute)
        self.d2h.wait_stream(compute)
        self._upload(0, batches[0])
        for i in range(len(batches)):
            slot = i % self.depth
            if i + 1 < len(batches):
                self._upload((i + 1) % self.depth, batches[i + 1])
            compute.wait_event(self.ready[slot])
            outs = step_fn(self.bufs[slot])
            done = torch.cuda.Event()
            done.record(compute)
            self.free[slot] = done
            if len(outs) != len(outputs[i]):
                raise ValueError("HostBatchPipeline: step_fn returned the wrong number of outputs")
            self.d2h.wait_event(done)
            with torch.cuda.stream(self.d2h):
                for src, dst in zip(outs, outputs[i]):
                    dst.copy_(src, non_blocking=True)
                    src.record_stream(self.d2h)
                    self.d2h_bytes += src.numel() * src.element_size()
        compute.wait_stream(self.d2h)
        compute.wait_stream(self.h2d)
