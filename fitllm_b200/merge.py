"""LoRA merge: bake the adapters into the frozen weights before inference.

FitLLM's ``merge_lora_into_shards`` (fitllm/inference.py:79-144) walks the
layer shard files once, and for every weight with a ``lora_A`` / ``lora_B``
pair in the same shard writes ``(W.float() + scale * (B @ A)).to(dtype)``
with ``scale = alpha / rank``, drops the adapter tensors and re-saves the
file with its checksum.  Here the per-weight step is one sm_100a kernel
(``fitq_lora_merge``, in place on the device).  Dense bf16 / fp16 weights
(and fp32) merge as the reference does.  An NF4 weight (the flat bitsandbytes key set)
is dequantised bit-exactly (in its compute dtype), merged and quantised again to NF4 with
the same level tables, so the shard keeps its format; that last step is a
new rounding of the merged weight, so the merged NF4 weight is not the
dense merge to the bit.
"""
from __future__ import annotations

from pathlib import Path
from typing import Dict, Iterable, List, Optional, Tuple

import torch

from . import _lib
from .nf4 import QuantState, dequantize_nf4, quantize_nf4
from .shards import load_shard_with_checksum, save_shard_with_checksum

_DTYPES = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16, torch.float32: _lib.DTYPE_F32}
_QS_KEYS = ("absmax", "quant_map", "nested_absmax", "nested_quant_map")


def lora_merge_(w: torch.Tensor, lora_a: torch.Tensor, lora_b: torch.Tensor, scale: float) -> torch.Tensor:
    """W <- W + scale * (B @ A) in place.  w: CUDA bf16/fp16/fp32 [N, K];
    lora_a [rank, K], lora_b [N, rank] (any float dtype; used as fp32)."""
    if not w.is_cuda:
        raise ValueError("lora_merge_ needs a CUDA weight")
    if w.dtype not in _DTYPES:
        raise ValueError(f"lora_merge_: weight dtype {w.dtype} is not bf16/fp16/fp32")
    if not w.is_contiguous():
        raise ValueError("lora_merge_: weight must be contiguous")
    n, k = w.shape
    a = lora_a.detach().to(w.device, torch.float32).contiguous()
    b = lora_b.detach().to(w.device, torch.float32).contiguous()
    rank = int(a.shape[0])
    if a.shape != (rank, k) or b.shape != (n, rank):
        raise ValueError(f"lora_merge_: A {tuple(a.shape)} / B {tuple(b.shape)} do not fit W [{n}, {k}]")
    L = _lib.load()
    with torch.cuda.device(w.device):
        _lib.check(L.fitq_lora_merge(w.data_ptr(), _DTYPES[w.dtype], n, k, a.data_ptr(), b.data_ptr(),
                                     rank, float(scale), torch.cuda.current_stream(w.device).cuda_stream),
                   "fitq_lora_merge")
    return w


def merge_nf4(packed: torch.Tensor, qs: QuantState, lora_a: torch.Tensor, lora_b: torch.Tensor,
              scale: float) -> Tuple[torch.Tensor, QuantState]:
    """NF4 weight + scale * (B @ A), re-quantised to NF4 with the same level
    tables: dequantise (bf16, bit-exact), merge in place, quantise."""
    w = dequantize_nf4(packed, qs, qs.dtype if qs.dtype in (torch.bfloat16, torch.float16) else torch.bfloat16)
    lora_merge_(w, lora_a, lora_b, scale)
    packed2, qs2 = quantize_nf4(w, qs.quant_map, qs.nested_quant_map, compute_dtype=qs.dtype)
    return packed2.view(packed.shape), qs2


def _lora_pair(tensors: Dict[str, torch.Tensor], module: str) -> Tuple[Optional[str], Optional[str]]:
    """The lora_A / lora_B keys of a module, found the way the reference does:
    any key containing "lora_A" (resp. "lora_B") and the module's last name."""
    short = module.split(".")[-1]
    a_key = b_key = None
    for k in tensors:
        if "lora_A" in k and short in k:
            a_key = k
        if "lora_B" in k and short in k:
            b_key = k
    return a_key, b_key


def _peft_layout(a: torch.Tensor, b: torch.Tensor, n: int, k: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """A [rank, K], B [N, rank] from the PEFT layout or FitLLM's own
    LoRALinear layout (lora_A [K, rank], lora_B [rank, N])."""
    if a.dim() == 2 and a.shape[1] == k and b.shape[0] == n:
        return a, b
    if a.dim() == 2 and a.shape[0] == k and b.shape[1] == n:
        return a.t(), b.t()
    raise ValueError(f"LoRA pair {tuple(a.shape)} / {tuple(b.shape)} does not fit a [{n}, {k}] weight")


def merge_shard_tensors(tensors: Dict[str, torch.Tensor], scale: float, device) -> List[str]:
    """Merge every adapter pair of one shard's tensors in place (dict
    updated, adapter keys removed).  Returns the merged weight keys."""
    merged = []
    for key in [k for k in tensors if k.endswith(".weight") and "lora_" not in k]:
        module = key[: -len(".weight")]
        a_key, b_key = _lora_pair(tensors, module)
        if a_key is None or b_key is None:
            continue
        w = tensors[key]
        qs_keys = {s: f"{key}.{s}" for s in _QS_KEYS if f"{key}.{s}" in tensors}
        if "absmax" in qs_keys:  # NF4 weight in the flat bitsandbytes key set
            flat = {s: tensors[k] for s, k in qs_keys.items()}
            for k in tensors:
                if k.startswith(f"{key}.quant_state."):
                    flat[k[len(key) + 1:]] = tensors[k]
            qs = QuantState.from_dict(flat, device=device)
            n, k = qs.shape
            a, b = _peft_layout(tensors[a_key], tensors[b_key], n, k)
            packed, qs2 = merge_nf4(w.to(device), qs, a, b, scale)
            tensors[key] = packed.cpu()
            for s, v in qs2.as_dict(packed=True).items():
                tensors[f"{key}.{s}"] = v.cpu() if isinstance(v, torch.Tensor) else v
        else:
            n, k = w.shape
            a, b = _peft_layout(tensors[a_key], tensors[b_key], n, k)
            wd = w.to(device, copy=True).contiguous()
            tensors[key] = lora_merge_(wd, a, b, scale).cpu()
        del tensors[a_key]
        del tensors[b_key]
        merged.append(key)
    return merged


def merge_lora_into_shards(shard_paths: Iterable, rank: int = 16, alpha: float = 32.0,
                           device=None) -> Dict[str, List[str]]:
    """merge_lora_into_shards (fitllm/inference.py:79-144) over shard files:
    scale = alpha / rank; each file is loaded, merged on the GPU and saved
    back with its checksum when it held an adapter.  Returns {path: merged
    weight keys}."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    scale = alpha / rank
    done: Dict[str, List[str]] = {}
    for path in shard_paths:
        path = Path(path)
        if not path.exists():
            continue
        tensors = load_shard_with_checksum(path, verify=False)
        merged = merge_shard_tensors(tensors, scale, dev)
        if merged:
            save_shard_with_checksum(tensors, path)
            done[str(path)] = merged
    return done
