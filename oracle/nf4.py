"""CPU oracle for the NF4 QLoRA path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
import this module, always as the checker.  The product package
(``fitllm_b200``) never imports it.

Two independent restatements live here and are checked against each other:

* the C oracle (``oracle/nf4_oracle.c``, loaded through ctypes), and
* a vectorised numpy restatement of the same arithmetic.

What they restate (reference behaviour, third-party code absent from the tree):

* ``bitsandbytes>=0.43.0`` (requirements.txt:19; unpinned, no lock file) supplies
  NF4 quantisation/dequantisation for FitLLM's ``BitsAndBytesConfig(load_in_4bit,
  nf4, double_quant=True)`` (fitllm/model.py:211-219).  Its QuantState is rebuilt
  from flat keys in fitllm/forward.py:76-109.
* NF4 levels: the 16 NormalFloat quantiles of Dettmers et al., "QLoRA" (2023),
  built from N(0,1) quantiles with offset 0.9677 (``normal_map_from_quantiles``
  rebuilds them from that published construction and must agree with
  ``NF4_LEVELS`` to fp32 rounding).
* Nested absmax codes: the signed 8-bit dynamic map of Dettmers et al., "8-bit
  Optimizers via Block-wise Quantization" (2022), ``dynamic_map_signed``.
* Dequant op order: absmax_b = fl(fl(nqm[code_b] * nabs[b//256]) + offset);
  w = fl(qm[nib] * absmax_b) rounded to bf16 (RNE).

Parity status: dequant op order pinned by call sites; quantiser parity-UNPINNED
against bitsandbytes (no bnb-produced vectors are reachable).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_LIB_PATH = HERE / "_build" / "libnf4_oracle.so"

NF4_BLOCK = 64
DQ_BLOCK = 256
OFFSET_CHUNK = 4096

# The 16 NF4 levels (QLoRA paper, Appendix E), as fp32.
NF4_LEVELS = np.array([
    -1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
    -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
    0.07958029955625534, 0.16093020141124725, 0.24611230194568634,
    0.33791524171829224, 0.44070982933044434, 0.5626170039176941,
    0.7229568362236023, 1.0], dtype=np.float32)


def normal_map_from_quantiles(offset: float = 0.9677083) -> np.ndarray:
    """Rebuild the NF4 levels from the published construction (QLoRA, 2023):
    8 positive quantiles of N(0,1) over linspace(offset, 0.5, 9)[:-1], 7 negative
    ones over linspace(offset, 0.5, 8)[:-1], plus an exact 0, normalised by the
    max.  Used only to pin ``NF4_LEVELS``."""
    from scipy.stats import norm
    pos = norm.ppf(np.linspace(offset, 0.5, 9)[:-1]).tolist()
    neg = (-norm.ppf(np.linspace(offset, 0.5, 8)[:-1])).tolist()
    v = np.array(sorted(pos + [0.0] + neg), dtype=np.float64)
    v = v / v.max()
    return v.astype(np.float32)


def dynamic_map_signed(max_exponent_bits: int = 7, total_bits: int = 8) -> np.ndarray:
    """Signed 8-bit dynamic quantisation map (Dettmers et al., 2022).

    For exponent i in 0..6 the interval [0.1, 1] is split into 2**i + 1 linearly
    spaced boundaries; the midpoints, scaled by 10**(i - 6), give 2**i positive
    and 2**i negative entries.  0 and 1.0 complete the 256 entries; the table is
    sorted ascending.  Computed with torch fp32 ops in that order so the values
    equal those of the published implementation's torch code.
    """
    import torch
    data = []
    non_sign_bits = total_bits - 1
    for i in range(max_exponent_bits):
        items = int(2 ** (i + non_sign_bits - max_exponent_bits) + 1)
        bounds = torch.linspace(0.1, 1, items)
        means = (bounds[:-1] + bounds[1:]) / 2.0
        scale = 10 ** (-(max_exponent_bits - 1) + i)
        data += (scale * means).tolist()
        data += (-scale * means).tolist()
    data.append(0)
    data.append(1.0)
    assert len(data) == 2 ** total_bits
    data.sort()
    return torch.tensor(data).numpy().astype(np.float32)


# ----------------------------------------------------------------------------
# C oracle through ctypes
# ----------------------------------------------------------------------------
_lib = None


def build() -> Path:
    """Compile oracle/nf4_oracle.c into oracle/_build/ (gcc, no FMA contraction)."""
    src = HERE / "nf4_oracle.c"
    if not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(_LIB_PATH))
        P, I64, F = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float
        L.oracle_nf4_quantize.argtypes = [P, I64, P, P, P]
        L.oracle_absmax_offset.argtypes = [P, I64]
        L.oracle_absmax_offset.restype = F
        L.oracle_dq_quantize.argtypes = [P, I64, P, F, P, P]
        L.oracle_absmax_decode.argtypes = [P, P, P, F, I64, P]
        L.oracle_nf4_dequant.argtypes = [P, P, P, P, P, F, I64, ctypes.c_int, P]
        L.oracle_nf4_dequant_plain.argtypes = [P, P, P, I64, ctypes.c_int, P]
        L.oracle_f32_to_bf16.argtypes = [F]
        L.oracle_f32_to_bf16.restype = ctypes.c_uint16
        L.oracle_f32_to_f16.argtypes = [F]
        L.oracle_f32_to_f16.restype = ctypes.c_uint16
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.c_void_p)


class NF4State:
    """Host-side copy of one quantised weight (the flat-key tensor set)."""

    def __init__(self, packed, absmax_code, nested_absmax, quant_map, nested_quant_map,
                 offset, shape):
        self.packed = packed                    # uint8 [N*K/2]
        self.absmax_code = absmax_code          # uint8 [N*K/64]
        self.nested_absmax = nested_absmax      # fp32  [ceil(N*K/64/256)]
        self.quant_map = quant_map              # fp32  [16]
        self.nested_quant_map = nested_quant_map  # fp32 [256]
        self.offset = np.float32(offset)
        self.shape = tuple(shape)


def quantize(w: np.ndarray, quant_map=None, nested_quant_map=None) -> NF4State:
    """C oracle: NF4 blockwise quantisation + double quantisation of absmax."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    n = w.size
    assert n % NF4_BLOCK == 0
    qm = NF4_LEVELS if quant_map is None else np.ascontiguousarray(quant_map, np.float32)
    nqm = dynamic_map_signed() if nested_quant_map is None else np.ascontiguousarray(nested_quant_map, np.float32)
    nb = n // NF4_BLOCK
    packed = np.empty(n // 2, np.uint8)
    absmax = np.empty(nb, np.float32)
    L = lib()
    L.oracle_nf4_quantize(_p(w), n, _p(qm), _p(packed), _p(absmax))
    offset = L.oracle_absmax_offset(_p(absmax), nb)
    nn = (nb + DQ_BLOCK - 1) // DQ_BLOCK
    codes = np.empty(nb, np.uint8)
    nabs = np.empty(nn, np.float32)
    L.oracle_dq_quantize(_p(absmax), nb, _p(nqm), ctypes.c_float(offset), _p(codes), _p(nabs))
    return NF4State(packed, codes, nabs, qm.copy(), nqm.copy(), offset, w.shape)


def absmax_decode(st: NF4State) -> np.ndarray:
    nb = st.absmax_code.size
    out = np.empty(nb, np.float32)
    lib().oracle_absmax_decode(_p(st.absmax_code), _p(st.nested_absmax), _p(st.nested_quant_map),
                               ctypes.c_float(st.offset), nb, _p(out))
    return out


def dequant(st: NF4State, out: str = "bf16") -> np.ndarray:
    """C oracle dequant.  Returns uint16 bit patterns for bf16/fp16, fp32 otherwise."""
    n = st.packed.size * 2
    kind = {"bf16": 0, "f16": 1, "f32": 2}[out]
    res = np.empty(n, np.uint16 if kind < 2 else np.float32)
    lib().oracle_nf4_dequant(_p(st.packed), _p(st.absmax_code), _p(st.nested_absmax),
                             _p(st.quant_map), _p(st.nested_quant_map), ctypes.c_float(st.offset),
                             n, kind, _p(res))
    return res.reshape(st.shape)


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Vectorised round-to-nearest-even fp32 -> bf16 bit patterns."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


# ----------------------------------------------------------------------------
# numpy restatement (independent of the C file; cross-checked in tests)
# ----------------------------------------------------------------------------
def _thresholds(levels: np.ndarray) -> np.ndarray:
    lv = levels.astype(np.float32)
    return (np.float32(0.5) * (lv[:-1] + lv[1:])).astype(np.float32)


def quantize_np(w: np.ndarray, quant_map=None, nested_quant_map=None) -> NF4State:
    w = np.ascontiguousarray(w, dtype=np.float32).reshape(-1)
    qm = NF4_LEVELS if quant_map is None else np.asarray(quant_map, np.float32)
    nqm = dynamic_map_signed() if nested_quant_map is None else np.asarray(nested_quant_map, np.float32)
    blocks = w.reshape(-1, NF4_BLOCK)
    absmax = np.abs(blocks).max(axis=1).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(absmax > 0, np.float32(1.0) / absmax, np.float32(0.0)).astype(np.float32)
    x = (blocks * inv[:, None]).astype(np.float32)
    codes4 = np.searchsorted(_thresholds(qm), x, side="left").astype(np.uint8).reshape(-1)
    packed = ((codes4[0::2] << 4) | codes4[1::2]).astype(np.uint8)
    nb = absmax.size
    total = 0.0
    for c in range(0, nb, OFFSET_CHUNK):
        # np.cumsum accumulates strictly left to right (np.sum is pairwise)
        total += float(np.cumsum(absmax[c:c + OFFSET_CHUNK].astype(np.float64))[-1])
    offset = np.float32(total / nb)
    centred = (absmax - offset).astype(np.float32)
    nn = (nb + DQ_BLOCK - 1) // DQ_BLOCK
    pad = np.zeros(nn * DQ_BLOCK, np.float32)
    pad[:nb] = np.abs(centred)
    nabs = pad.reshape(nn, DQ_BLOCK).max(axis=1).astype(np.float32)
    with np.errstate(divide="ignore"):
        ninv = np.where(nabs > 0, np.float32(1.0) / nabs, np.float32(0.0)).astype(np.float32)
    xn = (centred * np.repeat(ninv, DQ_BLOCK)[:nb]).astype(np.float32)
    codes8 = np.searchsorted(_thresholds(nqm), xn, side="left").astype(np.uint8)
    return NF4State(packed, codes8, nabs, qm.copy(), nqm.copy(), offset, (w.size,))


def dequant_np(st: NF4State) -> np.ndarray:
    """numpy restatement of the dequant; returns bf16 bit patterns."""
    nb = st.absmax_code.size
    p = (st.nested_quant_map[st.absmax_code] *
         np.repeat(st.nested_absmax, DQ_BLOCK)[:nb]).astype(np.float32)
    am = (p + np.float32(st.offset)).astype(np.float32)
    hi = st.packed >> 4
    lo = st.packed & 0x0F
    nib = np.empty(st.packed.size * 2, np.uint8)
    nib[0::2] = hi
    nib[1::2] = lo
    v = (st.quant_map[nib] * np.repeat(am, NF4_BLOCK)).astype(np.float32)
    return f32_to_bf16_bits(v).reshape(st.shape)


def dequant_torch(st: NF4State):
    """The dequant of ``dequant_np`` in torch CPU ops (all host threads): the
    same two rounded fp32 operations per block and one per weight, then RNE to
    bf16.  Returns fp32 values [shape] (exactly bf16-representable)."""
    import torch
    codes = torch.from_numpy(st.absmax_code).long()
    nb = codes.numel()
    nabs = torch.from_numpy(st.nested_absmax).repeat_interleave(DQ_BLOCK)[:nb]
    am = torch.from_numpy(st.nested_quant_map)[codes] * nabs + torch.tensor(st.offset)
    packed = torch.from_numpy(st.packed)
    nib = torch.stack(((packed >> 4) & 0x0F, packed & 0x0F), dim=1).reshape(-1).long()
    w = torch.from_numpy(st.quant_map)[nib].view(nb, NF4_BLOCK) * am[:, None]
    return w.to(torch.bfloat16).float().reshape(st.shape)


# ----------------------------------------------------------------------------
# QLoRA linear reference math (fp64 on the exact bf16-valued inputs)
# ----------------------------------------------------------------------------
def qlora_forward(x: np.ndarray, w: np.ndarray, A: np.ndarray, B: np.ndarray, s: float) -> np.ndarray:
    """Y = x.W^T + s.(x.A^T).B^T  (PEFT lora.Linear4bit with dropout inactive).

    x [M,K], w [N,K] (dequantised), A [r,K], B [N,r]."""
    x64, w64, A64, B64 = (np.asarray(t, np.float64) for t in (x, w, A, B))
    return x64 @ w64.T + s * (x64 @ A64.T) @ B64.T


def qlora_backward(x, w, A, B, s, dy):
    """Returns (dX, dA, dB) of the QLoRA linear for upstream grad dy [M,N].

    T = x.A^T; U = dy.B; dB = s.dy^T.T; dA = s.U^T.x; dX = dy.W + s.U.A"""
    x64, w64, A64, B64, dy64 = (np.asarray(t, np.float64) for t in (x, w, A, B, dy))
    T = x64 @ A64.T
    U = dy64 @ B64
    dB = s * dy64.T @ T
    dA = s * U.T @ x64
    dX = dy64 @ w64 + s * U @ A64
    return dX, dA, dB


def rel_err(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))
