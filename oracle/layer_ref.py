"""CPU restatement of one shard-stationary QLoRA layer step -- TEST / BASELINE
INFRASTRUCTURE ONLY (tests, __graft_entry__.smoke and bench.py's CPU legs).

What it restates: FitLLM's per-layer work in a training step
(fitllm/forward.py:480-528 forward without autograd, then
fitllm/backward.py:206-249 recompute-with-autograd + backward) for a
Qwen2.5-32B-shaped decoder layer whose projections are NF4 (bitsandbytes
dequant arithmetic, via the C oracle) with PEFT LoRA on q/v (dropout inactive),
computed in fp32 on the host cores with torch CPU ops.
"""
from __future__ import annotations

import math
import os
import time
from typing import Dict, Tuple

import numpy as np
import torch
import torch.nn.functional as F

from . import nf4 as onf4

PROJ = [("q_proj", "q", True), ("k_proj", "kv", True), ("v_proj", "kv", True),
        ("o_proj", "o", False), ("gate_proj", "i", False), ("up_proj", "i", False),
        ("down_proj", "d", False)]


def proj_shape(kind: str, hidden: int, heads: int, kv_heads: int, head_dim: int, inter: int):
    return {"q": (heads * head_dim, hidden), "kv": (kv_heads * head_dim, hidden),
            "o": (hidden, heads * head_dim), "i": (inter, hidden), "d": (hidden, inter)}[kind]


def build_layer(hidden=5120, heads=40, kv_heads=8, head_dim=128, inter=27648, rank=16,
                alpha=32.0, seed=0) -> Dict[str, torch.Tensor]:
    """Seeded N(0,0.02) weights -> NF4 (C oracle) -> dequantised fp32 weights
    (the exact bf16 values bitsandbytes' dequant produces), plus LoRA A/B."""
    w = {}
    g = torch.Generator().manual_seed(seed)
    for name, kind, bias in PROJ:
        n, k = proj_shape(kind, hidden, heads, kv_heads, head_dim, inter)
        dense = (torch.randn(n, k, generator=g) * 0.02).numpy()
        st = onf4.quantize(dense)
        w[name] = torch.from_numpy(onf4.bf16_bits_to_f32(onf4.dequant(st, "bf16")))
        if bias:
            w[name + ".bias"] = (torch.randn(n, generator=g) * 0.02).bfloat16().float()
    for name in ("q_proj", "v_proj"):
        n, k = w[name].shape
        w[name + ".lora_A"] = (torch.rand(rank, k, generator=g) * 2 - 1) / math.sqrt(k)
        w[name + ".lora_B"] = torch.randn(n, rank, generator=g) * 0.01
    w["scale"] = torch.tensor(alpha / rank)
    w["cfg"] = torch.tensor([hidden, heads, kv_heads, head_dim, inter])
    return w


def _rms(x, eps=1e-6):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)


def _rope(seq, head_dim, theta=1e6, device=None, dtype=torch.float32):
    """HF rotary tables (cos, sin) [S, head_dim], computed in fp32 and cast to
    the activations' dtype (as Qwen2RotaryEmbedding returns them)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    f = torch.outer(torch.arange(seq, dtype=torch.float32), inv)
    e = torch.cat([f, f], -1)
    return e.cos().to(device, dtype), e.sin().to(device, dtype)


def _rot(x):
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), -1)


def layer_forward(w, h):
    """One decoder layer in the dtype and on the device of h and w (fp32 on
    the host cores for the oracle; bf16 on a GPU restates the reference's own
    precision: bf16 activations, fp32-accumulating matmuls)."""
    hidden, heads, kv_heads, head_dim, inter = [int(v) for v in w["cfg"]]
    s = float(w["scale"])
    b, S, _ = h.shape

    def lin(name, x):
        y = x @ w[name].T
        if name + ".bias" in w:
            y = y + w[name + ".bias"]
        if name + ".lora_A" in w:
            y = y + s * (x @ w[name + ".lora_A"].T) @ w[name + ".lora_B"].T
        return y

    x = _rms(h)
    q = lin("q_proj", x).view(b, S, heads, head_dim).transpose(1, 2)
    k = lin("k_proj", x).view(b, S, kv_heads, head_dim).transpose(1, 2)
    v = lin("v_proj", x).view(b, S, kv_heads, head_dim).transpose(1, 2)
    cos, sin = _rope(S, head_dim, device=h.device, dtype=h.dtype)
    q, k = q * cos + _rot(q) * sin, k * cos + _rot(k) * sin
    o = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
    h1 = h + lin("o_proj", o.transpose(1, 2).reshape(b, S, heads * head_dim))
    x2 = _rms(h1)
    return h1 + lin("down_proj", F.silu(lin("gate_proj", x2)) * lin("up_proj", x2))


def layer_step(w, h, grad_out) -> Tuple[torch.Tensor, Dict[str, torch.Tensor]]:
    """Shard-stationary per-layer work: forward (no autograd), recompute with
    autograd, backward.  Returns (grad wrt h, LoRA grads)."""
    with torch.no_grad():
        layer_forward(w, h)
    params = {k: w[k].clone().requires_grad_(True) for k in w if "lora_" in k}
    ww = dict(w)
    ww.update(params)
    x = h.clone().requires_grad_(True)
    y = layer_forward(ww, x)
    y.backward(grad_out)
    return x.grad, {k: p.grad for k, p in params.items()}


_LAYER_CACHE: Dict[int, Dict[str, torch.Tensor]] = {}


def _cached_layer(seed: int) -> Dict[str, torch.Tensor]:
    if seed not in _LAYER_CACHE:
        _LAYER_CACHE[seed] = build_layer(seed=seed)
    return _LAYER_CACHE[seed]


def time_cpu_step(seq=2048, microbatches=1, seed=0, threads=None) -> Dict[str, float]:
    """Time one layer step on the host cores; returns tokens/s and details."""
    threads = threads or os.cpu_count()
    torch.set_num_threads(threads)
    t0 = time.perf_counter()
    w = _cached_layer(seed)
    t_build = time.perf_counter() - t0
    g = torch.Generator().manual_seed(seed + 5)
    hidden = int(w["cfg"][0])
    h = torch.randn(microbatches, seq, hidden, generator=g).bfloat16().float()
    go = torch.randn(microbatches, seq, hidden, generator=g).bfloat16().float()
    t0 = time.perf_counter()
    layer_step(w, h, go)
    dt = time.perf_counter() - t0
    return {"tokens_per_s": microbatches * seq / dt, "step_s": dt, "threads": threads,
            "quantize_s": t_build, "tokens": microbatches * seq}


# ----------------------------------------------------------------------------
# CPU baselines of the other workloads (timed on the host cores, all threads)
# ----------------------------------------------------------------------------
def time_cpu_qproj(m=512, n=5120, k=5120, r=16, alpha=32.0, threads=None) -> Dict[str, float]:
    """One NF4 QLoRA q_proj linear, forward + backward (dX, dA, dB), in fp32
    torch on the host cores: the oracle-dequantised weight (untimed), PEFT
    LoRA (A Kaiming-uniform [r, K], B N(0, 0.01) [N, r]), x and dY N(0, 1)."""
    threads = threads or os.cpu_count()
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    st = onf4.quantize((torch.randn(n, k, generator=g) * 0.02).numpy())
    w = onf4.dequant_torch(st)
    A = ((torch.rand(r, k, generator=g) * 2 - 1) / math.sqrt(k)).requires_grad_(True)
    B = (torch.randn(n, r, generator=g) * 0.01).requires_grad_(True)
    x = torch.randn(m, k, generator=g).bfloat16().float().requires_grad_(True)
    dy = torch.randn(m, n, generator=g).bfloat16().float()
    s = alpha / r

    def call():
        A.grad = B.grad = x.grad = None
        y = x @ w.T + s * (x @ A.T) @ B.T
        y.backward(dy)

    call()
    t0 = time.perf_counter()
    reps = 3
    for _ in range(reps):
        call()
    dt = (time.perf_counter() - t0) / reps
    return {"tokens_per_s": m / dt, "call_s": dt, "threads": threads,
            "tflops": m * (4 * n * k + 6 * r * (n + k)) / dt / 1e12}


def time_cpu_gemv(n, k, m, r=0, threads=None) -> Dict[str, float]:
    """One NF4 GEMV call on the host cores: dequant of the weight (torch ops,
    the oracle's op order) + the [m, K] x [K, N] product (+ LoRA), fp32."""
    threads = threads or os.cpu_count()
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(n + k)
    st = onf4.quantize((torch.randn(n, k, generator=g) * 0.02).numpy())
    x = torch.randn(m, k, generator=g).bfloat16().float()
    A = torch.randn(r, k, generator=g) * 0.01 if r else None
    B = torch.randn(n, r, generator=g) * 0.01 if r else None

    def call():
        w = onf4.dequant_torch(st)
        y = x @ w.T
        if r:
            y = y + 2.0 * (x @ A.T) @ B.T
        return y

    call()
    t0 = time.perf_counter()
    reps = 2
    for _ in range(reps):
        call()
    dt = (time.perf_counter() - t0) / reps
    wbytes = n * k // 2 + n * k // 64 + ((n * k // 64 + 255) // 256) * 4
    return {"us": dt * 1e6, "GB/s": wbytes / dt / 1e9, "threads": threads}


def time_cpu_verify_layer(batch=8, t_new=5, prefix=4096, seed=0, threads=None) -> Dict[str, float]:
    """One decoder layer of a KV-cached speculative-verify pass on the host
    cores (fp32 torch): the batch x t_new new tokens through the projections
    (oracle-dequantised NF4 weights, LoRA on q/v), RoPE at positions prefix..,
    attention of token i over cache positions <= prefix + i (GQA), MLP.  The
    64-layer pass time is 64 x this layer's (stated as extrapolated)."""
    threads = threads or os.cpu_count()
    torch.set_num_threads(threads)
    w = _cached_layer(seed)
    hidden, heads, kv_heads, head_dim, inter = [int(v) for v in w["cfg"]]
    s = float(w["scale"])
    g = torch.Generator().manual_seed(seed + 9)
    h = torch.randn(batch, t_new, hidden, generator=g).bfloat16().float()
    L = prefix + t_new
    kc = torch.randn(batch, kv_heads, L, head_dim, generator=g).bfloat16().float()
    vc = torch.randn(batch, kv_heads, L, head_dim, generator=g).bfloat16().float()

    def lin(name, x):
        y = x @ w[name].T
        if name + ".bias" in w:
            y = y + w[name + ".bias"]
        if name + ".lora_A" in w:
            y = y + s * (x @ w[name + ".lora_A"].T) @ w[name + ".lora_B"].T
        return y

    def call():
        x = _rms(h)
        q = lin("q_proj", x).view(batch, t_new, heads, head_dim).transpose(1, 2)
        k = lin("k_proj", x).view(batch, t_new, kv_heads, head_dim).transpose(1, 2)
        v = lin("v_proj", x).view(batch, t_new, kv_heads, head_dim).transpose(1, 2)
        cos, sin = _rope(L, head_dim)
        cos, sin = cos[prefix:], sin[prefix:]
        q, k = q * cos + _rot(q) * sin, k * cos + _rot(k) * sin
        kc[:, :, prefix:] = k
        vc[:, :, prefix:] = v
        pos = torch.arange(L)
        lim = prefix + torch.arange(t_new)
        mask = pos[None, :] <= lim[:, None]
        o = F.scaled_dot_product_attention(q, kc, vc, attn_mask=mask, enable_gqa=True)
        h1 = h + lin("o_proj", o.transpose(1, 2).reshape(batch, t_new, heads * head_dim))
        x2 = _rms(h1)
        return h1 + lin("down_proj", F.silu(lin("gate_proj", x2)) * lin("up_proj", x2))

    with torch.no_grad():
        call()
        t0 = time.perf_counter()
        reps = 3
        for _ in range(reps):
            call()
        dt = (time.perf_counter() - t0) / reps
    return {"layer_s": dt, "pass_s_64_layers": 64 * dt,
            "tokens_per_s": batch * t_new / (64 * dt), "threads": threads}
