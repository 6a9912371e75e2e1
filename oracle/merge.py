"""CPU restatement of the LoRA merge -- TEST INFRASTRUCTURE ONLY (tests).

What it restates: the per-weight step of FitLLM's merge_lora_into_shards
(fitllm/inference.py:127-131): W_merged = (W.float() + scale * (B @ A)) cast
back to W's dtype, scale = alpha / rank (fitllm/inference.py:110-112), with
A = lora_A [rank, K] and B = lora_B [N, rank].  The reference leaves the
order of the rank sum to torch's CPU matmul; this restatement fixes it to
rank order with every fp32 product and partial sum rounded (numpy float32
arithmetic), the order the device kernel uses, so the two agree bit for
bit; `reference_formula` is the reference's own torch expression, which
the tests hold this restatement to within one rounding of the output dtype.
"""
from __future__ import annotations

import numpy as np
import torch

from . import nf4 as onf4


def rank_sum(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """(B @ A) in fp32, rank ascending, each product and sum rounded."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    t = np.zeros((b.shape[0], a.shape[1]), np.float32)
    for j in range(a.shape[0]):
        t = (t + (b[:, j:j + 1] * a[j:j + 1, :])).astype(np.float32)
    return t


def merge_f32(w: np.ndarray, a: np.ndarray, b: np.ndarray, scale: float) -> np.ndarray:
    """fl(W + fl(scale * t)) in fp32 (W given as fp32 values)."""
    t = rank_sum(a, b)
    return (np.asarray(w, np.float32) + (np.float32(scale) * t).astype(np.float32)).astype(np.float32)


def merge_bf16_bits(w_bits: np.ndarray, a, b, scale: float) -> np.ndarray:
    """bf16 W (bit patterns) -> merged bf16 bit patterns (round to nearest even)."""
    return onf4.f32_to_bf16_bits(merge_f32(onf4.bf16_bits_to_f32(w_bits), a, b, scale))


def merge_f16(w: np.ndarray, a, b, scale: float) -> np.ndarray:
    return merge_f32(np.asarray(w, np.float16).astype(np.float32), a, b, scale).astype(np.float16)


def reference_formula(w: torch.Tensor, a: torch.Tensor, b: torch.Tensor, scale: float) -> torch.Tensor:
    """fitllm/inference.py:128-131 as written: (W.float() + scale * (B @ A)).to(W.dtype)."""
    return (w.float() + scale * (b.float() @ a.float())).to(w.dtype)
