"""Micro-batch data parallelism inside a layer (one process per GPU).

FitLLM itself is single-device (no torch.distributed anywhere; the patent text
claims single-GPU operation, FitLLM_Patent_v8.md:340).  On a B200 box the
grad_accum micro-batches of each layer are split across the ranks; each rank
runs the shard-stationary forward/backward on its share, and the only exchange
is ONE all-reduce (sum, fp32) of that layer's LoRA gradients, issued as soon as
the layer's backward is queued so that it overlaps the next layer's backward.
Every rank then applies the identical optimizer step, so adapters stay equal
bit for bit.
"""
from __future__ import annotations

import datetime
import os
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist


def microbatch_range(num_microbatches: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous share [start, stop) of the micro-batches for `rank`.

    Shares differ by at most one when world does not divide the count."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, extra = divmod(num_microbatches, world)
    start = rank * base + min(rank, extra)
    stop = start + base + (1 if rank < extra else 0)
    return start, stop


def init_from_env(backend: Optional[str] = None, timeout_s: float = 300.0) -> Tuple[int, int]:
    """Initialise the default process group from torchrun's environment
    (127.0.0.1 rendezvous).  Returns (rank, world); (0, 1) when not launched
    under torchrun."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world <= 1:
        return 0, 1
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        kw = {}
        if backend == "nccl":
            kw["device_id"] = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return dist.get_rank(), dist.get_world_size()


class LoRAGradComm:
    """Per-layer asynchronous all-reduce of a LoRAStore's gradient slices."""

    def __init__(self, store, group=None):
        self.store = store
        self.group = group
        self._pending: List = []
        self.enabled = dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1

    def allreduce_layer(self, layer: int) -> None:
        if not self.enabled:
            return
        buf = self.store.layer_slice(self.store.grad, layer)
        self._pending.append(dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=self.group,
                                             async_op=True))

    def wait(self) -> None:
        for h in self._pending:
            h.wait()
        self._pending.clear()


def barrier(group=None) -> None:
    if dist.is_available() and dist.is_initialized():
        if torch.cuda.is_available() and dist.get_backend(group) == "nccl":
            dist.barrier(group=group, device_ids=[torch.cuda.current_device()])
        else:
            dist.barrier(group=group)


def max_over_ranks(value: float, device=None) -> float:
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
