"""NF4 weights in the bitsandbytes Params4bit / QuantState format.

FitLLM loads its layers with ``BitsAndBytesConfig(load_in_4bit=True,
bnb_4bit_quant_type="nf4", bnb_4bit_use_double_quant=True)``
(fitllm/model.py:211-219) and, after every shard load, rebuilds each
weight's QuantState from the flat keys ``<param>``, ``.absmax``,
``.quant_map``, ``.nested_absmax``, ``.nested_quant_map`` and
``.quant_state.bitsandbytes__nf4`` (fitllm/forward.py:76-109).  This module
holds that tensor set on the device and runs the sm_100a quantise/dequantise
kernels on it through the C ABI.
"""
from __future__ import annotations

import ctypes
import json
from dataclasses import dataclass, field
from typing import Dict, Optional, Tuple

import torch

from . import _lib

BLOCKSIZE = 64
NESTED_BLOCKSIZE = 256

# NF4 levels (Dettmers et al., QLoRA 2023): the 16 normal-quantile code values.
NF4_LEVELS = (
    -1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
    -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
    0.07958029955625534, 0.16093020141124725, 0.24611230194568634,
    0.33791524171829224, 0.44070982933044434, 0.5626170039176941,
    0.7229568362236023, 1.0)


def nf4_quant_map(device=None) -> torch.Tensor:
    return torch.tensor(NF4_LEVELS, dtype=torch.float32, device=device)


def dynamic_quant_map(device=None) -> torch.Tensor:
    """Signed 8-bit dynamic map (Dettmers et al., "8-bit Optimizers via
    Block-wise Quantization", 2022) used for the nested absmax codes: for
    i = 0..6, the midpoints of linspace(0.1, 1, 2**i + 1) scaled by 10**(i-6),
    positive and negative, plus 0 and 1.0, sorted ascending."""
    vals = []
    for i in range(7):
        b = torch.linspace(0.1, 1, 2 ** i + 1)
        mid = (b[:-1] + b[1:]) / 2.0
        s = 10 ** (i - 6)
        vals += (s * mid).tolist()
        vals += (-s * mid).tolist()
    vals += [0, 1.0]
    vals.sort()
    return torch.tensor(vals, dtype=torch.float32, device=device)


_DTYPE_NAMES = {torch.bfloat16: "bfloat16", torch.float16: "float16", torch.float32: "float32"}
_NAME_DTYPES = {v: k for k, v in _DTYPE_NAMES.items()}


@dataclass
class QuantState:
    """The QuantState fields the NF4 kernels consume (nested = double quant)."""
    absmax: torch.Tensor                    # uint8 codes (nested) or fp32 (plain), [N*K/64]
    shape: Tuple[int, int]                  # (N, K)
    quant_map: torch.Tensor                 # fp32 [16]
    dtype: torch.dtype = torch.bfloat16     # compute dtype
    blocksize: int = BLOCKSIZE
    quant_type: str = "nf4"
    nested_absmax: Optional[torch.Tensor] = None      # fp32 [ceil(N*K/64/256)]
    nested_quant_map: Optional[torch.Tensor] = None   # fp32 [256]
    offset: float = 0.0
    nested_blocksize: int = NESTED_BLOCKSIZE
    _keep: list = field(default_factory=list, repr=False)

    @property
    def nested(self) -> bool:
        return self.nested_absmax is not None

    # --- bitsandbytes serialisation (flat keys under "<param>.") -------------
    def as_dict(self, packed: bool = True) -> Dict[str, torch.Tensor]:
        d = {"absmax": self.absmax, "quant_map": self.quant_map}
        meta = {
            "quant_type": self.quant_type,
            "blocksize": self.blocksize,
            "dtype": _DTYPE_NAMES.get(self.dtype, "bfloat16"),
            "shape": list(self.shape),
        }
        if self.nested:
            d["nested_absmax"] = self.nested_absmax
            d["nested_quant_map"] = self.nested_quant_map
            meta.update({"nested_blocksize": self.nested_blocksize, "nested_dtype": "float32",
                         "nested_offset": float(self.offset)})
        if packed:
            raw = json.dumps(meta).encode("utf-8")
            d["quant_state.bitsandbytes__" + self.quant_type] = torch.tensor(list(raw), dtype=torch.uint8)
        else:
            d.update(meta)
        return d

    @classmethod
    def from_dict(cls, qs: Dict[str, torch.Tensor], device=None) -> "QuantState":
        """Inverse of as_dict; accepts the packed-JSON key like
        bitsandbytes' QuantState.from_dict does."""
        qs = dict(qs)
        meta = {}
        for k in list(qs):
            if k.startswith("quant_state.bitsandbytes__"):
                meta = json.loads(bytes(qs.pop(k).cpu().tolist()).decode("utf-8"))
        for k in ("quant_type", "blocksize", "dtype", "shape", "nested_blocksize", "nested_dtype",
                  "nested_offset"):
            if k in qs and k not in meta:
                meta[k] = qs.pop(k)
        if meta.get("quant_type", "nf4") != "nf4":
            raise ValueError("only NF4 quantisation is supported")
        dev = torch.device(device) if device is not None else qs["absmax"].device
        nested = "nested_absmax" in qs
        shape = tuple(int(s) for s in meta["shape"])
        return cls(
            absmax=qs["absmax"].to(dev),
            shape=(shape[0], shape[1]) if len(shape) == 2 else (shape[0], 1),
            quant_map=qs["quant_map"].to(dev, torch.float32),
            dtype=_NAME_DTYPES.get(str(meta.get("dtype", "bfloat16")).replace("torch.", ""), torch.bfloat16),
            blocksize=int(meta.get("blocksize", BLOCKSIZE)),
            nested_absmax=qs["nested_absmax"].to(dev, torch.float32) if nested else None,
            nested_quant_map=qs["nested_quant_map"].to(dev, torch.float32) if nested else None,
            offset=float(meta.get("nested_offset", 0.0)),
            nested_blocksize=int(meta.get("nested_blocksize", NESTED_BLOCKSIZE)),
        )

    def to(self, device) -> "QuantState":
        f = lambda t: None if t is None else t.to(device, non_blocking=True)
        return QuantState(f(self.absmax), self.shape, f(self.quant_map), self.dtype, self.blocksize,
                          self.quant_type, f(self.nested_absmax), f(self.nested_quant_map),
                          self.offset, self.nested_blocksize)


def weight_struct(packed: torch.Tensor, qs: QuantState) -> Nf4WeightCRef:
    return Nf4WeightCRef(packed, qs)


class Nf4WeightCRef:
    """struct fitq_nf4_weight for one weight (keeps the tensors alive)."""

    def __init__(self, packed: torch.Tensor, qs: QuantState):
        if qs.blocksize != BLOCKSIZE:
            raise ValueError(f"NF4 blocksize {qs.blocksize} unsupported (kernels use 64)")
        if qs.nested and qs.nested_blocksize != NESTED_BLOCKSIZE:
            raise ValueError("nested blocksize must be 256")
        n, k = qs.shape
        if packed.numel() * 2 != n * k:
            raise ValueError(f"packed has {packed.numel()} bytes, shape {qs.shape} needs {n * k // 2}")
        self.tensors = (packed, qs.absmax, qs.nested_absmax, qs.nested_quant_map, qs.quant_map)
        self.c = _lib.Nf4WeightC(
            packed=packed.data_ptr(),
            absmax_code=qs.absmax.data_ptr() if qs.nested else None,
            nested_absmax=qs.nested_absmax.data_ptr() if qs.nested else None,
            nested_quant_map=qs.nested_quant_map.data_ptr() if qs.nested else None,
            absmax_f32=None if qs.nested else qs.absmax.data_ptr(),
            quant_map=qs.quant_map.data_ptr(),
            offset=float(qs.offset), n_out=n, k_in=k)

    @property
    def ref(self):
        return ctypes.byref(self.c)


def _stream(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def quantize_nf4(w: torch.Tensor, quant_map: Optional[torch.Tensor] = None,
                 nested_quant_map: Optional[torch.Tensor] = None,
                 compute_dtype: torch.dtype = torch.bfloat16) -> Tuple[torch.Tensor, QuantState]:
    """Quantise a CUDA weight W[N, K] to NF4 with double-quantised absmax.

    Returns (packed uint8 [N*K/2, 1], QuantState) like bitsandbytes'
    quantize_4bit(..., quant_type="nf4", compress_statistics=True)."""
    if not w.is_cuda:
        raise ValueError("quantize_nf4 needs a CUDA tensor")
    n, k = w.shape
    dev = w.device
    w32 = w.detach().to(torch.float32).contiguous()
    qm = nf4_quant_map(dev) if quant_map is None else quant_map.to(dev, torch.float32).contiguous()
    nqm = dynamic_quant_map(dev) if nested_quant_map is None else nested_quant_map.to(dev, torch.float32).contiguous()
    nb = n * k // BLOCKSIZE
    packed = torch.empty(n * k // 2, 1, dtype=torch.uint8, device=dev)
    codes = torch.empty(nb, dtype=torch.uint8, device=dev)
    nabs = torch.empty((nb + NESTED_BLOCKSIZE - 1) // NESTED_BLOCKSIZE, dtype=torch.float32, device=dev)
    off = torch.empty(1, dtype=torch.float32, device=dev)
    L = _lib.load()
    ws_bytes = L.fitq_nf4_quantize_workspace(n, k)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _lib.check(L.fitq_nf4_quantize(w32.data_ptr(), n, k, qm.data_ptr(), nqm.data_ptr(),
                                       packed.data_ptr(), codes.data_ptr(), nabs.data_ptr(),
                                       off.data_ptr(), ws.data_ptr(), ws_bytes, _stream(dev)),
                   "fitq_nf4_quantize")
    qs = QuantState(absmax=codes, shape=(n, k), quant_map=qm, dtype=compute_dtype,
                    nested_absmax=nabs, nested_quant_map=nqm, offset=float(off.item()))
    return packed, qs


def dequantize_nf4(packed: torch.Tensor, qs: QuantState, out_dtype: torch.dtype = torch.bfloat16,
                   transpose: bool = False) -> torch.Tensor:
    """Bit-exact dequantisation (bitsandbytes dequantize_4bit op order)."""
    n, k = qs.shape
    code = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16}[out_dtype]
    out = torch.empty((k, n) if transpose else (n, k), dtype=out_dtype, device=packed.device)
    ws = Nf4WeightCRef(packed, qs)
    L = _lib.load()
    with torch.cuda.device(packed.device):
        _lib.check(L.fitq_nf4_dequant(ws.ref, out.data_ptr(), code, int(transpose),
                                      _stream(packed.device)), "fitq_nf4_dequant")
    return out
