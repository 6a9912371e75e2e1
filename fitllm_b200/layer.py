"""Qwen2.5-32B-shaped decoder layer whose seven projections are NF4.

The layer FitLLM drives through its shard-stationary loop is a HuggingFace
``Qwen2DecoderLayer`` after QLoRA preparation (fitllm/model.py:209-267,
fitllm/forward.py:657-701): RMSNorm, q/k/v (with bias) / o projections,
RoPE (theta 1e6), causal GQA attention (40 query / 8 KV heads of 128),
RMSNorm, SwiGLU MLP (27648).  This module keeps HF's attribute names
(``self_attn.q_proj``, ``mlp.gate_proj``, ``input_layernorm`` ...) so the
shard keys of fitllm/forward.py:95-109 load unchanged, and runs:

* every projection as an NF4 ``Linear4bit`` / ``QLoRALinear4bit`` on the
  sm_100a kernels (the residual adds of o_proj and down_proj ride in the GEMM
  epilogue);
* RMSNorm and the rotary embedding as fused one-pass kernels of the same
  library (layer_ops.cu); gate/up as one GEMM with SwiGLU in its epilogue and
  the SwiGLU backward in down_proj's dX epilogue; attention with torch SDPA
  (library kernel).
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field
from typing import Optional, Sequence, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from .layer_ops import attention, rms_norm, rope, swiglu
from .qlora import Linear4bit, QLoRALinear4bit


@dataclass
class LayerConfig:
    hidden: int = 5120
    heads: int = 40
    kv_heads: int = 8
    head_dim: int = 128
    intermediate: int = 27648
    rms_eps: float = 1e-6
    rope_theta: float = 1e6
    vocab: int = 152064
    lora_rank: int = 16
    lora_alpha: float = 32.0
    lora_targets: Tuple[str, ...] = ("q_proj", "v_proj")

    @classmethod
    def qwen25_32b(cls, **kw) -> "LayerConfig":
        return cls(**kw)

    def proj_shapes(self):
        """(name, N_out, K_in, has_bias) of the seven projections."""
        h, q, kv, i = self.hidden, self.heads * self.head_dim, self.kv_heads * self.head_dim, self.intermediate
        return [("self_attn.q_proj", q, h, True), ("self_attn.k_proj", kv, h, True),
                ("self_attn.v_proj", kv, h, True), ("self_attn.o_proj", h, q, False),
                ("mlp.gate_proj", i, h, False), ("mlp.up_proj", i, h, False),
                ("mlp.down_proj", h, i, False)]

    def nf4_weights_per_layer(self) -> int:
        return sum(n * k for _, n, k, _ in self.proj_shapes())


class RMSNorm(nn.Module):
    """Qwen2RMSNorm: fp32 variance, weight applied after casting back."""

    def __init__(self, hidden: int, eps: float, device=None, dtype=torch.bfloat16):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden, device=device, dtype=dtype), requires_grad=False)
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return rms_norm(x, self.weight, self.eps)


def rotary_cos_sin(seq_len: int, head_dim: int, theta: float, device, dtype=torch.bfloat16,
                   position_ids: Optional[torch.Tensor] = None):
    """(cos, sin) [S, head_dim] of the HF rotary embedding (rotate_half layout)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=device, dtype=torch.float32) / head_dim))
    pos = torch.arange(seq_len, device=device, dtype=torch.float32) if position_ids is None \
        else position_ids.to(device, torch.float32)
    freqs = torch.outer(pos, inv)
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def rotary_tables(seq_len: int, head_dim: int, theta: float, device,
                  position_ids: Optional[torch.Tensor] = None):
    """fp32 (cos, sin) [S, head_dim/2] of the rotary frequencies (the fused
    kernel duplicates them over the two halves, as HF's cat([f, f]) does)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=device, dtype=torch.float32) / head_dim))
    pos = torch.arange(seq_len, device=device, dtype=torch.float32) if position_ids is None \
        else position_ids.to(device, torch.float32)
    f = torch.outer(pos, inv)
    return f.cos().contiguous(), f.sin().contiguous()


def _as_half_tables(pe, head_dim):
    cos, sin = pe
    if cos.shape[-1] == head_dim:  # HF-style full (cos, sin): keep the first half in fp32
        cos, sin = cos[..., : head_dim // 2], sin[..., : head_dim // 2]
    if cos.dim() == 3:
        cos, sin = cos[0], sin[0]
    return cos.float().contiguous(), sin.float().contiguous()


def _rotate_half(x):
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def apply_rotary(q, k, cos, sin):
    # q: [B, H, S, D]; cos/sin: [S, D]
    return q * cos + _rotate_half(q) * sin, k * cos + _rotate_half(k) * sin


class Attention(nn.Module):
    def __init__(self, cfg: LayerConfig, device=None):
        super().__init__()
        self.cfg = cfg
        h, qd, kvd = cfg.hidden, cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
        self.q_proj = Linear4bit(h, qd, bias=True, device=device)
        self.k_proj = Linear4bit(h, kvd, bias=True, device=device)
        self.v_proj = Linear4bit(h, kvd, bias=True, device=device)
        self.o_proj = Linear4bit(qd, h, bias=False, device=device)
        # FITQ_ATTN=1: this library's causal GQA attention kernels (fwd + bwd,
        # [B, S, heads, 128] in place, no transposes) instead of torch SDPA.
        self.own_kernel = os.environ.get("FITQ_ATTN", "0") == "1"

    def forward(self, x, residual, cos, sin, attn_mask: Optional[torch.Tensor] = None):
        cfg = self.cfg
        b, s, _ = x.shape
        if (self.own_kernel and attn_mask is None and x.is_cuda and cfg.head_dim == 128
                and s % 64 == 0):
            q = rope(self.q_proj(x), cos, sin, cfg.heads).view(b, s, cfg.heads, cfg.head_dim)
            k = rope(self.k_proj(x), cos, sin, cfg.kv_heads).view(b, s, cfg.kv_heads, cfg.head_dim)
            v = self.v_proj(x).view(b, s, cfg.kv_heads, cfg.head_dim)
            o = attention(q, k, v).view(b, s, cfg.heads * cfg.head_dim)
            return self.o_proj(o, residual=residual)
        q = rope(self.q_proj(x), cos, sin, cfg.heads).view(b, s, cfg.heads, cfg.head_dim).transpose(1, 2)
        k = rope(self.k_proj(x), cos, sin, cfg.kv_heads).view(b, s, cfg.kv_heads, cfg.head_dim).transpose(1, 2)
        v = self.v_proj(x).view(b, s, cfg.kv_heads, cfg.head_dim).transpose(1, 2)
        if attn_mask is None:
            o = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
        else:
            o = F.scaled_dot_product_attention(q, k, v, attn_mask=attn_mask, enable_gqa=True)
        o = o.transpose(1, 2).reshape(b, s, cfg.heads * cfg.head_dim)
        return self.o_proj(o, residual=residual)


class _FusedMLPFn(torch.autograd.Function):
    """out = down(silu(gate(x)) * up(x)) + residual with plain NF4 projections.

    Forward: gate and up as one GEMM whose epilogue applies the SwiGLU, then
    down_proj with the residual in its epilogue.  Backward: down_proj's dX
    GEMM applies the SwiGLU backward in its epilogue (d_gate, d_up), then the
    gate and up dX GEMMs accumulate into one dx.  Bit-identical to the
    separate projections + SwiGLU kernels (same GEMMs, same epilogue math)."""

    @staticmethod
    def forward(ctx, x, residual, wg, wu, wd, bwd_fused=True):
        from . import ops
        lead = x.shape[:-1]
        x2 = ops._bf16_2d(x, wg.c.k_in)
        keep = ctx.needs_input_grad[0]
        act, gate, up = ops.nf4_gateup_swiglu(x2, wg, wu, keep_gate_up=keep)
        res2 = ops._bf16_2d(residual, wd.c.n_out)
        y, _ = ops.qlora_forward(act, wd, None, None, 1.0, y_add=res2)
        ctx.refs = (wg, wu, wd)
        ctx.lead = lead
        ctx.bwd_fused = bwd_fused
        ctx.save_for_backward(gate, up)
        return y.view(*lead, wd.c.n_out)

    @staticmethod
    def backward(ctx, dy):
        from . import ops
        gate, up = ctx.saved_tensors
        wg, wu, wd = ctx.refs
        dy2 = ops._bf16_2d(dy, wd.c.n_out)
        dx = None
        if ctx.needs_input_grad[0]:
            if ctx.bwd_fused:
                d_gate, d_up = ops.nf4_down_dswiglu(dy2, wd, gate, up)
            else:  # down_proj dX, then the separate SwiGLU backward kernel
                from .layer_ops import swiglu_backward
                d_act, _, _ = ops.qlora_backward(None, dy2, wd, None, None, 1.0)
                d_gate, d_up = swiglu_backward(d_act, gate, up)
            dx, _, _ = ops.qlora_backward(None, d_gate, wg, None, None, 1.0)
            ops.qlora_backward(None, d_up, wu, None, None, 1.0, dx=dx)
            dx = dx.view(*ctx.lead, wg.c.k_in)
        dres = dy if ctx.needs_input_grad[1] else None
        return dx, dres, None, None, None, None


def _plain_nf4(mod) -> bool:
    return isinstance(mod, Linear4bit) and mod.bias is None and mod.quant_state is not None


class MLP(nn.Module):
    def __init__(self, cfg: LayerConfig, device=None):
        super().__init__()
        self.gate_proj = Linear4bit(cfg.hidden, cfg.intermediate, device=device)
        self.up_proj = Linear4bit(cfg.hidden, cfg.intermediate, device=device)
        self.down_proj = Linear4bit(cfg.intermediate, cfg.hidden, device=device)
        # FITQ_MLP_FUSED=1: gate/up + SwiGLU in one GEMM, SwiGLU backward in
        # down's dX; FITQ_MLP_FUSED=fwd: the forward fusion only.  Off by
        # default: on a power-capped B200 the Qwen2.5-32B layer step measured
        # 3-6% slower with both (the fused GEMMs ran at a lower SM clock)
        # although they remove three element-wise passes.
        mode = os.environ.get("FITQ_MLP_FUSED", "0")
        self.fused = mode in ("1", "fwd")
        self.fused_backward = mode == "1"

    def forward(self, x, residual):
        if (self.fused and x.is_cuda and _plain_nf4(self.gate_proj) and _plain_nf4(self.up_proj)
                and _plain_nf4(self.down_proj) and self.gate_proj.out_features % 128 == 0):
            return _FusedMLPFn.apply(x, residual, self.gate_proj.wref(), self.up_proj.wref(),
                                     self.down_proj.wref(), self.fused_backward)
        return self.down_proj(swiglu(self.gate_proj(x), self.up_proj(x)), residual=residual)


class DecoderLayer(nn.Module):
    """h_out = h + o_proj(attn(norm(h)));  out = h_out + down(silu(gate) * up)(norm(h_out))."""

    def __init__(self, cfg: LayerConfig, device=None):
        super().__init__()
        self.cfg = cfg
        self.input_layernorm = RMSNorm(cfg.hidden, cfg.rms_eps, device=device)
        self.self_attn = Attention(cfg, device=device)
        self.post_attention_layernorm = RMSNorm(cfg.hidden, cfg.rms_eps, device=device)
        self.mlp = MLP(cfg, device=device)

    def forward(self, h: torch.Tensor, position_embeddings=None, attention_mask=None, **_):
        if position_embeddings is None:
            position_embeddings = rotary_tables(h.shape[1], self.cfg.head_dim, self.cfg.rope_theta,
                                                h.device)
        cos, sin = _as_half_tables(position_embeddings, self.cfg.head_dim)
        h1 = self.self_attn(self.input_layernorm(h), h, cos, sin, attention_mask)
        return self.mlp(self.post_attention_layernorm(h1), h1)

    def projections(self):
        for name, _, _, _ in self.cfg.proj_shapes():
            yield name, self.get_submodule(name)

    def lora_modules(self):
        for name, mod in self.projections():
            if isinstance(mod, QLoRALinear4bit):
                yield name, mod


def quantize_layer_(layer: DecoderLayer, seed: int, std: float = 0.02,
                    bias_std: float = 0.02) -> None:
    """Fill every projection with NF4 weights quantised on the device from
    seeded N(0, std) fp32 values (biases N(0, bias_std) in bf16)."""
    dev = layer.input_layernorm.weight.device
    g = torch.Generator(device=dev)
    for i, (name, n, k, has_bias) in enumerate(layer.cfg.proj_shapes()):
        mod = layer.get_submodule(name)
        base = mod.base_layer if isinstance(mod, QLoRALinear4bit) else mod
        g.manual_seed(seed * 100 + i)
        w = torch.randn(n, k, generator=g, device=dev, dtype=torch.float32) * std
        fresh = Linear4bit.from_float(w, None)
        del w
        base.set_quantized(fresh.weight.data, fresh.quant_state)
        if has_bias:
            base.bias.data.copy_((torch.randn(n, generator=g, device=dev) * bias_std).to(base.bias.dtype))


def add_lora_(layer: DecoderLayer, rank: int, alpha: float, targets: Sequence[str], seed: int,
              b_std: float = 0.0) -> None:
    """Wrap the target projections with rank-r adapters (PEFT init: A
    Kaiming-uniform, B zeros, or N(0, b_std) when b_std > 0 so that dA != 0)."""
    for i, (name, mod) in enumerate(list(layer.projections())):
        short = name.rsplit(".", 1)[-1]
        if short in targets and isinstance(mod, Linear4bit):
            parent = layer.get_submodule(name.rsplit(".", 1)[0])
            torch.manual_seed(seed * 1000 + i)
            q = QLoRALinear4bit(mod, r=rank, lora_alpha=alpha)
            if b_std > 0:
                with torch.no_grad():
                    q.lora_B["default"].weight.normal_(0.0, b_std)
            setattr(parent, short, q)
