"""KV-cached speculative-verify forward over NF4 QLoRA layers.

FitLLM verifies draft tokens by re-running the full prefix through the model
(fitllm/inference.py:380-397, the prefill path of fitllm/forward.py:547-655).
This module runs the same layers over a key/value cache instead: each verify
step feeds only the draft + 1 new tokens of every sequence (batch B, T tokens
each), so every projection is a skinny NF4 GEMM with M = B * T rows (the
decode kernels of this library), attention reads the cached prefix, and the
new keys/values are written into the cache at positions [P, P + T).

The layer arithmetic is DecoderLayer's (fitllm_b200/layer.py): RMSNorm, q/k/v
with bias, rotary embedding at the tokens' absolute positions, grouped-query
attention (causal within the new tokens, full over the prefix), o_proj with
the residual fused, RMSNorm, SwiGLU MLP with the residual fused.

Attention runs on the library's split-KV kernel (fitq_verify_attention) when
head_dim is 128 and (heads / kv_heads) * T <= 32 -- every verify step of the
Qwen2.5 shapes; other shapes (e.g. filling a cache with a long prompt) use
torch's scaled_dot_product_attention with the prefix + causal mask.
"""
from __future__ import annotations

from typing import List, Tuple

import torch
import torch.nn.functional as F

from . import ops
from .layer import DecoderLayer, rotary_tables
from .layer_ops import rope_kv_append, swiglu
from .qlora import QLoRALinear4bit, grouped_forward, swiglu_forward


class KVCache:
    """Per-layer key/value cache [B, kv_heads, capacity, head_dim] (bf16)."""

    def __init__(self, num_layers: int, batch: int, kv_heads: int, head_dim: int, capacity: int,
                 device, dtype=torch.bfloat16):
        shape = (batch, kv_heads, capacity, head_dim)
        self.k = [torch.zeros(shape, device=device, dtype=dtype) for _ in range(num_layers)]
        self.v = [torch.zeros(shape, device=device, dtype=dtype) for _ in range(num_layers)]
        self.capacity = capacity

    def fill_random_(self, length: int, seed: int = 0) -> None:
        """Seeded N(0, 1) prefix of `length` positions (a synthetic context)."""
        g = torch.Generator(device=self.k[0].device).manual_seed(seed)
        for k, v in zip(self.k, self.v):
            k[:, :, :length].normal_(generator=g)
            v[:, :, :length].normal_(generator=g)

    def bytes_read(self, length: int) -> int:
        """K and V bytes one verify pass reads over `length` cached positions."""
        b, h, _, d = self.k[0].shape
        return 2 * len(self.k) * b * h * length * d * self.k[0].element_size()


def verify_mask(prefix: int, t: int, device) -> torch.Tensor:
    """[t, prefix + t] boolean: new token i sees the prefix and new tokens <= i."""
    cols = torch.arange(prefix + t, device=device)
    rows = torch.arange(t, device=device)
    return cols[None, :] <= (prefix + rows)[:, None]


def kernel_attention_ok(cfg, t: int) -> bool:
    """Shapes fitq_verify_attention covers: head_dim 128, (heads / kv_heads) * t <= 32."""
    return cfg.head_dim == 128 and (cfg.heads // cfg.kv_heads) * t <= 32


def verify_layer_forward(layer: DecoderLayer, h: torch.Tensor, k_cache: torch.Tensor,
                         v_cache: torch.Tensor, prefix: int, tables: Tuple[torch.Tensor, torch.Tensor],
                         mask: torch.Tensor) -> torch.Tensor:
    """One layer over the T new tokens of each sequence.  h: [B, T, hidden]
    bf16; tables: fp32 rotary (cos, sin) half tables of positions
    [prefix, prefix + T); writes K/V of the new tokens into the caches."""
    cfg = layer.cfg
    b, t, _ = h.shape
    attn = layer.self_attn
    cos, sin = tables
    x = layer.input_layernorm(h)
    grouped = b * t <= 64  # the skinny GEMM path: q/k/v (and gate/up) as one launch each
    if grouped:
        q_raw, k_raw, v_raw = grouped_forward([attn.q_proj, attn.k_proj, attn.v_proj], x)
    else:
        q_raw, k_raw, v_raw = attn.q_proj(x), attn.k_proj(x), attn.v_proj(x)
    # rotary embedding of q and k and the append of k, v to the caches: one launch
    q = rope_kv_append(q_raw, k_raw, v_raw, cos, sin, k_cache, v_cache, prefix, cfg.heads,
                       cfg.kv_heads)
    if kernel_attention_ok(cfg, t):
        o = ops.verify_attention(q, k_cache, v_cache, prefix)
    else:
        o = F.scaled_dot_product_attention(q.transpose(1, 2), k_cache[:, :, :prefix + t],
                                           v_cache[:, :, :prefix + t], attn_mask=mask,
                                           enable_gqa=True).transpose(1, 2)
    o = o.reshape(b, t, cfg.heads * cfg.head_dim)
    h1 = attn.o_proj(o, residual=h)
    mlp = layer.mlp
    x2 = layer.post_attention_layernorm(h1)
    if grouped and not isinstance(mlp.gate_proj, QLoRALinear4bit) and not isinstance(mlp.up_proj,
                                                                                       QLoRALinear4bit):
        act = swiglu_forward(mlp.gate_proj, mlp.up_proj, x2)  # gate/up/SwiGLU, one GEMM + one finish
    else:
        gate, up = grouped_forward([mlp.gate_proj, mlp.up_proj], x2) if grouped else (
            mlp.gate_proj(x2), mlp.up_proj(x2))
        act = swiglu(gate, up)
    return mlp.down_proj(act, residual=h1)


@torch.no_grad()
def verify_pass(layers: List[DecoderLayer], h: torch.Tensor, cache: KVCache, prefix: int) -> torch.Tensor:
    """All layers over the new tokens; returns the final hidden states."""
    cfg = layers[0].cfg
    t = h.shape[1]
    pos = torch.arange(prefix, prefix + t, device=h.device)
    tables = rotary_tables(t, cfg.head_dim, cfg.rope_theta, h.device, position_ids=pos)
    mask = None if kernel_attention_ok(cfg, t) else verify_mask(prefix, t, h.device)
    for i, layer in enumerate(layers):
        h = verify_layer_forward(layer, h, cache.k[i], cache.v[i], prefix, tables, mask)
    return h
