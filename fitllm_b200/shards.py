"""Layer shard files: safetensors + SHA-256 sidecar -> pinned host arena.

FitLLM keeps one safetensors file per decoder layer,
``layer_{i:03d}_weights.safetensors`` (``layer_{a:03d}-{b:03d}_weights.safetensors``
with ``"{offset}."`` key prefixes when ``shard_group_size > 1``), written by
``shard_model`` (fitllm/model.py:25-83) through ``save_shard_with_checksum``
(fitllm/scheduler.py:21-27), which also writes the file's hex SHA-256 to a
``.sha256`` sidecar.  Every read goes through ``load_shard_with_checksum``
(fitllm/scheduler.py:30-59), re-hashing the whole file before use when
verification is on (fitllm/scheduler.py:347-384).

Here the files have the same names, keys and sidecars, but a shard is read
and verified ONCE, when its layer enters the pinned host store of
``ShardScheduler`` (the copy the device ring streams from on every pass);
the steady-state loop never touches the file system.  Hashing runs in a
thread pool (hashlib releases the GIL on large updates), so loading N layers
overlaps their checksums.
"""
from __future__ import annotations

import hashlib
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path
from typing import Dict, Iterable, List, Optional, Tuple

import torch

_CHUNK = 1 << 22


def compute_file_sha256(path) -> str:
    """Hex SHA-256 of a file (fitllm/scheduler.py:62-67)."""
    h = hashlib.sha256()
    with open(path, "rb") as f:
        while True:
            b = f.read(_CHUNK)
            if not b:
                break
            h.update(b)
    return h.hexdigest()


def checksum_path(path) -> Path:
    return Path(path).with_suffix(".sha256")


def save_shard_with_checksum(state_dict: Dict[str, torch.Tensor], path) -> None:
    """Write a safetensors shard and its ``.sha256`` sidecar (fitllm/scheduler.py:21-27)."""
    from safetensors.torch import save_file
    path = Path(path)
    save_file({k: v.detach().contiguous().cpu() for k, v in state_dict.items()}, str(path))
    checksum_path(path).write_text(compute_file_sha256(path))


def verify_shard(path) -> None:
    """Raise RuntimeError when the sidecar exists and does not match the file."""
    path = Path(path)
    side = checksum_path(path)
    if not side.exists():
        return
    expected = side.read_text().strip()
    actual = compute_file_sha256(path)
    if actual != expected:
        raise RuntimeError(f"Checksum mismatch for shard {path}. Expected {expected}, got {actual}. "
                           "The file may be corrupted.")


def load_shard_with_checksum(path, verify: bool = True) -> Dict[str, torch.Tensor]:
    """All tensors of a shard (CPU), after the checksum check when ``verify``
    (fitllm/scheduler.py:30-59: same error on a mismatch, no check without a sidecar)."""
    from safetensors import safe_open
    path = Path(path)
    if verify:
        verify_shard(path)
    out: Dict[str, torch.Tensor] = {}
    with safe_open(str(path), framework="pt", device="cpu") as f:
        for k in f.keys():
            out[k] = f.get_tensor(k)
    return out


def shard_file_name(first: int, last: Optional[int] = None) -> str:
    """``layer_{i:03d}_weights.safetensors`` for one layer per file (last None);
    ``layer_{a:03d}-{b:03d}_weights.safetensors`` for a group, even a group of
    one (fitllm/model.py:63-66 names by group size, not by group length)."""
    if last is None:
        return f"layer_{first:03d}_weights.safetensors"
    return f"layer_{first:03d}-{last:03d}_weights.safetensors"


def shard_groups(num_layers: int, group_size: int = 1) -> List[Tuple[int, int]]:
    """(first, last) layer of every file, as shard_model groups them."""
    if group_size < 1:
        raise ValueError("group_size must be >= 1")
    return [(a, min(a + group_size, num_layers) - 1) for a in range(0, num_layers, group_size)]


def write_layer_shards(layer_state_dicts: Iterable[Dict[str, torch.Tensor]], shard_dir,
                       group_size: int = 1) -> int:
    """Write per-layer state dicts as shard files (fitllm/model.py:25-83 layout).
    Returns the number of layers written."""
    if group_size < 1:
        raise ValueError("group_size must be >= 1")
    shard_dir = Path(shard_dir)
    shard_dir.mkdir(parents=True, exist_ok=True)
    group: Dict[str, torch.Tensor] = {}
    first = count = 0

    def flush(last: int) -> None:
        save_shard_with_checksum(group, shard_dir / shard_file_name(first, last if group_size > 1 else None))
        group.clear()

    # one group at a time, copied out: a producer may reuse its tensors for the next layer
    for n, sd in enumerate(layer_state_dicts):
        count = n + 1
        off = n - first
        for k, v in sd.items():
            group[k if group_size == 1 else f"{off}.{k}"] = v.detach().to("cpu", copy=True)
        if off == group_size - 1:
            flush(n)
            first = n + 1
    if group:
        flush(count - 1)
    return count


def split_group(tensors: Dict[str, torch.Tensor], count: int) -> List[Dict[str, torch.Tensor]]:
    """Per-layer dicts of a group file (keys ``"{offset}.{key}"``)."""
    out: List[Dict[str, torch.Tensor]] = [dict() for _ in range(count)]
    for k, v in tensors.items():
        off, _, rest = k.partition(".")
        out[int(off)][rest] = v
    return out


def load_shards_into(scheduler, shard_dir, num_layers: int, group_size: int = 1,
                     verify_checksums: bool = True, threads: int = 8) -> int:
    """Read every shard file once into ``scheduler``'s pinned host store
    (``ShardScheduler.add_layer``), checksums verified in parallel first.
    Returns the host bytes stored."""
    shard_dir = Path(shard_dir)
    groups = shard_groups(num_layers, group_size)
    paths = [shard_dir / shard_file_name(a, b if group_size > 1 else None) for a, b in groups]
    missing = [p for p in paths if not p.exists()]
    if missing:
        raise FileNotFoundError(f"Shard not found: {missing[0]}")
    if verify_checksums:
        with ThreadPoolExecutor(max_workers=max(1, threads)) as ex:
            list(ex.map(verify_shard, paths))
    total = 0
    for (first, last), path in zip(groups, paths):
        tensors = load_shard_with_checksum(path, verify=False)
        per_layer = [tensors] if group_size == 1 else split_group(tensors, last - first + 1)
        for off, t in enumerate(per_layer):
            total += scheduler.add_layer(first + off, t)
    return total
