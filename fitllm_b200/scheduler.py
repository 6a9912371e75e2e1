"""Shard upload path: pinned host store -> copy stream -> K-slot device ring.

Replaces the per-tensor ``.to(device, non_blocking)`` upload of
``ShardScheduler._transfer_to_gpu`` / ``get_layer_tensors``
(fitllm/scheduler.py:162-178, :259-290) and its per-eviction
``empty_cache``/``gc`` (fitllm/scheduler.py:317-324, :440-456), following the
resident-pinned-weights design the reference documents for itself
(EFFICIENT_TRAINING.md:81-193):

* every layer's shard (the flat key set of fitllm/forward.py:95-109) lives in
  ONE pinned host arena, each tensor at a 256-byte aligned offset;
* ``prefetch(l)`` issues one ``cudaMemcpyAsync`` of the whole arena on a
  dedicated copy stream into ring slot ``l % K`` once the compute stream has
  released that slot (event), so layer l+1 uploads while layer l computes;
* ``get_layer_tensors(l)`` makes the compute stream wait on the slot's ready
  event and returns device views with the same keys -- no allocation, no
  cache eviction, no synchronisation in the loop.

LoRA keys found in a shard are dropped, as fitllm/forward.py:733-734 does.

Data-parallel ranks (``group`` with more than one rank, NCCL): every rank
needs the whole layer, but PCIe is per GPU while NVLink is shared by all, so
by default each rank uploads only its 1/G byte range of the arena into its
part of the slot and one in-place NCCL all-gather over NVLink fills in the
rest (``shard_upload=False`` restores the replicated upload).  A rank then
needs only that byte range in host memory, so it pins just its 1/G of every
layer (``store_full=True`` keeps whole arenas, e.g. to compare against).
"""
from __future__ import annotations

import json
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch
import torch.distributed as dist

_ALIGN = 256


@dataclass
class _Entry:
    key: str
    offset: int
    nbytes: int
    dtype: torch.dtype
    shape: Tuple[int, ...]


def _layout(tensors: Dict[str, torch.Tensor]) -> Tuple[List[_Entry], int]:
    entries, off = [], 0
    for k in sorted(tensors):
        t = tensors[k]
        off = (off + _ALIGN - 1) // _ALIGN * _ALIGN
        nb = t.numel() * t.element_size()
        entries.append(_Entry(k, off, nb, t.dtype, tuple(t.shape)))
        off += nb
    return entries, (off + _ALIGN - 1) // _ALIGN * _ALIGN


def shard_ranges(total: int, world: int) -> Tuple[int, List[Tuple[int, int]]]:
    """Per-rank byte ranges [start, stop) of an arena of `total` bytes split over
    `world` ranks in equal 256-byte aligned chunks (the last ones may be short
    or empty).  Returns (chunk, ranges); chunk * world >= total."""
    if world < 1:
        raise ValueError("world must be >= 1")
    chunk = -(-max(total, 1) // world)
    chunk = (chunk + _ALIGN - 1) // _ALIGN * _ALIGN
    ranges = [(min(i * chunk, total), min((i + 1) * chunk, total)) for i in range(world)]
    return chunk, ranges


def _views(buf: torch.Tensor, entries: List[_Entry]) -> Dict[str, torch.Tensor]:
    out = {}
    for e in entries:
        raw = buf[e.offset:e.offset + e.nbytes]
        out[e.key] = raw.view(e.dtype).view(e.shape) if e.nbytes else torch.empty(e.shape, dtype=e.dtype, device=buf.device)
    return out


class ShardScheduler:
    """Pinned host store + device staging ring for layer shards."""

    def __init__(self, num_layers: int, device, ring_slots: int = 2, pin_memory: bool = True,
                 group=None, shard_upload: bool = True, store_full: bool = False):
        if ring_slots < 1:
            raise ValueError("ring_slots must be >= 1")
        self.group = group
        multi = dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1
        self.shard_upload = bool(shard_upload and multi)
        self.rank = dist.get_rank(group) if multi else 0
        self.world = dist.get_world_size(group) if multi else 1
        self.num_layers = num_layers
        self.device = torch.device(device)
        self.ring_slots = ring_slots
        self.pin_memory = pin_memory
        self.store_full = bool(store_full or not self.shard_upload)
        self._host: Dict[int, torch.Tensor] = {}   # pinned arena, or this rank's byte range of it
        self._total: Dict[int, int] = {}           # full arena bytes per layer
        self._layout: Dict[int, List[_Entry]] = {}
        self._meta: Dict[int, Dict[str, dict]] = {}
        self._slot_bytes = 0
        self._slots: List[Optional[torch.Tensor]] = [None] * ring_slots
        self._slot_layer: List[int] = [-1] * ring_slots
        self._ready: List[Optional[torch.cuda.Event]] = [None] * ring_slots
        self._free: List[Optional[torch.cuda.Event]] = [None] * ring_slots
        self._generation = 0  # slot map offset (advanced by invalidate)
        self._copy_stream: Optional[torch.cuda.Stream] = None
        self.h2d_bytes = 0

    # ---------------------------------------------------------------- host side
    def add_layer(self, layer_idx: int, tensors: Dict[str, torch.Tensor]) -> int:
        """Copy one layer's flat key set into its pinned host arena.  Returns bytes."""
        base = {k: v for k, v in tensors.items() if "lora_A" not in k and "lora_B" not in k}
        meta = {}
        for k in list(base):
            if k.endswith("quant_state.bitsandbytes__nf4"):
                meta[k[: -len(".quant_state.bitsandbytes__nf4")]] = json.loads(
                    bytes(base[k].cpu().tolist()).decode("utf-8"))
        entries, total = _layout(base)
        if self.store_full:
            arena = torch.zeros(total, dtype=torch.uint8, pin_memory=self.pin_memory)  # padding 0
            views = _views(arena, entries)
            for k, t in base.items():
                views[k].copy_(t.detach().cpu().view(views[k].dtype).view(views[k].shape))
        else:
            # assemble the arena where the tensors live, keep only this rank's range
            src_dev = next(iter(base.values())).device if base else torch.device("cpu")
            full = torch.zeros(total, dtype=torch.uint8, device=src_dev)
            views = _views(full, entries)
            for k, t in base.items():
                views[k].copy_(t.detach().view(views[k].dtype).view(views[k].shape))
            _, ranges = shard_ranges(total, self.world)
            a, b = ranges[self.rank]
            arena = torch.empty(b - a, dtype=torch.uint8, pin_memory=self.pin_memory)
            arena.copy_(full[a:b])
            del full, views
        self._host[layer_idx] = arena
        self._total[layer_idx] = total
        self._layout[layer_idx] = entries
        self._meta[layer_idx] = meta
        self._slot_bytes = max(self._slot_bytes, total)
        return total

    def layer_bytes(self, layer_idx: int) -> int:
        return int(self._total[layer_idx])

    def host_bytes(self) -> int:
        """Pinned host bytes this rank holds for all layers."""
        return int(sum(t.numel() for t in self._host.values()))

    def upload_bytes(self, layer_idx: int) -> int:
        """Bytes this rank copies host -> device for one layer."""
        total = self.layer_bytes(layer_idx)
        if not self.shard_upload:
            return total
        _, ranges = shard_ranges(total, self.world)
        a, b = ranges[self.rank]
        return b - a

    def host_tensors(self, layer_idx: int) -> Dict[str, torch.Tensor]:
        if not self.store_full:
            raise RuntimeError("this rank holds only its byte range of the layer (store_full=False)")
        return _views(self._host[layer_idx], self._layout[layer_idx])

    def quant_meta(self, layer_idx: int) -> Dict[str, dict]:
        """Parsed ``<param>.quant_state.bitsandbytes__nf4`` metadata (host, no sync)."""
        return self._meta[layer_idx]

    # ---------------------------------------------------------------- device ring
    def _ensure_ring(self):
        if self._copy_stream is None:
            self._copy_stream = torch.cuda.Stream(device=self.device)
        need = self._slot_bytes
        if self.shard_upload:  # room for world equal chunks of the largest arena
            chunk, _ = shard_ranges(self._slot_bytes, self.world)
            need = chunk * self.world
        for s in range(self.ring_slots):
            if self._slots[s] is None or self._slots[s].numel() < need:
                self._slots[s] = torch.empty(need, dtype=torch.uint8, device=self.device)
                self._slot_layer[s] = -1
                self._ready[s] = torch.cuda.Event()
                self._free[s] = None

    def slot_of(self, layer_idx: int) -> int:
        return (layer_idx + self._generation) % self.ring_slots

    def prefetch(self, layer_idx: int) -> None:
        """Start the async upload of a layer into its ring slot (idempotent)."""
        if layer_idx < 0 or layer_idx >= self.num_layers:
            return
        self._ensure_ring()
        s = self.slot_of(layer_idx)
        if self._slot_layer[s] == layer_idx:
            return
        cs = self._copy_stream
        if self._free[s] is not None:
            cs.wait_event(self._free[s])
        else:  # slot never released: wait for everything queued so far
            cs.wait_stream(torch.cuda.current_stream(self.device))
        self._free[s] = None
        src = self._host[layer_idx]
        with torch.cuda.stream(cs):
            if self.shard_upload:
                chunk, ranges = shard_ranges(self._total[layer_idx], self.world)
                a, b = ranges[self.rank]
                if b > a:
                    part = src[a:b] if self.store_full else src
                    self._slots[s][a:b].copy_(part, non_blocking=True)
                mine = self._slots[s][self.rank * chunk:(self.rank + 1) * chunk]
                # in place: this rank's chunk is already in position inside the output
                dist.all_gather_into_tensor(self._slots[s][: chunk * self.world], mine,
                                            group=self.group)
                self.h2d_bytes += b - a
            else:
                self._slots[s][: src.numel()].copy_(src, non_blocking=True)
                self.h2d_bytes += src.numel()
            self._ready[s].record(cs)
        self._slot_layer[s] = layer_idx

    def get_layer_tensors(self, layer_idx: int, verify_checksums: bool = False) -> Dict[str, torch.Tensor]:
        """Device views of the layer's tensors; the current stream waits for the upload."""
        self.prefetch(layer_idx)
        s = self.slot_of(layer_idx)
        torch.cuda.current_stream(self.device).wait_event(self._ready[s])
        return _views(self._slots[s], self._layout[layer_idx])

    def release(self, layer_idx: int) -> None:
        """Mark the slot reusable once the work queued so far on the current stream is done."""
        s = self.slot_of(layer_idx)
        if self._slot_layer[s] != layer_idx:
            return
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self._free[s] = ev

    def invalidate(self) -> None:
        """Forget which layers the ring holds, so the next get re-uploads.

        The slot map advances by one, so with two or more slots the next
        upload of a layer lands in a different slot than the one the work
        queued so far may still read: a caller can invalidate and prefetch
        the next step's first layer right after queueing the current step,
        and that upload overlaps the current step's work."""
        self._slot_layer = [-1] * self.ring_slots
        self._generation += 1

    def wait_uploads(self) -> None:
        """Make the current stream wait for every upload queued so far."""
        if self._copy_stream is not None:
            torch.cuda.current_stream(self.device).wait_stream(self._copy_stream)

    # reference-compatible names
    def prefetch_to_cpu(self, layer_idx: int, verify_checksums: bool = False) -> None:
        """The host store is resident; warm the device ring instead."""
        self.prefetch(layer_idx)

    def evict_layer_from_gpu(self, layer_idx: int) -> None:
        self.release(layer_idx)

    def synchronize(self) -> None:
        if self._copy_stream is not None:
            self._copy_stream.synchronize()
