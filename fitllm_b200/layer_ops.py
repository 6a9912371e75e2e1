"""Autograd wrappers of the fused decoder-layer kernels (RMSNorm, rotary
embedding, SwiGLU) that surround the QLoRA projections.  CUDA bf16 only."""
from __future__ import annotations

import torch

from . import _lib


def _st(t) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _c(t: torch.Tensor) -> torch.Tensor:
    return t if t.is_contiguous() else t.contiguous()


class RMSNormFn(torch.autograd.Function):
    """Qwen2RMSNorm with frozen weight: y = w * bf16(x * rsqrt(mean(x^2) + eps))."""

    @staticmethod
    def forward(ctx, x, weight, eps: float):
        x = _c(x)
        cols = x.shape[-1]
        rows = x.numel() // cols
        y = torch.empty_like(x)
        L = _lib.load()
        with torch.cuda.device(x.device):
            _lib.check(L.fitq_rmsnorm_fwd(x.data_ptr(), weight.data_ptr(), y.data_ptr(), rows, cols,
                                          float(eps), _st(x)), "fitq_rmsnorm_fwd")
        ctx.save_for_backward(x, weight)
        ctx.eps = eps
        return y

    @staticmethod
    def backward(ctx, dy):
        x, weight = ctx.saved_tensors
        dy = _c(dy.to(x.dtype))
        cols = x.shape[-1]
        rows = x.numel() // cols
        dx = torch.empty_like(x)
        L = _lib.load()
        with torch.cuda.device(x.device):
            _lib.check(L.fitq_rmsnorm_bwd(dy.data_ptr(), x.data_ptr(), weight.data_ptr(), dx.data_ptr(),
                                          rows, cols, float(ctx.eps), _st(x)), "fitq_rmsnorm_bwd")
        return dx, None, None


class RoPEFn(torch.autograd.Function):
    """Rotate-half rotary embedding of t [B, S, heads*head_dim] (bf16) with fp32
    half tables cos/sin [S, head_dim/2]; returns a new tensor of t's shape."""

    @staticmethod
    def forward(ctx, t, cos_half, sin_half, heads: int):
        t = _c(t)
        seq = t.shape[-2]
        dim = t.shape[-1] // heads
        rows = t.numel() // (heads * dim)
        out = torch.empty_like(t)
        L = _lib.load()
        with torch.cuda.device(t.device):
            _lib.check(L.fitq_rope(t.data_ptr(), out.data_ptr(), cos_half.data_ptr(), sin_half.data_ptr(),
                                   rows, heads, dim, seq, 0, _st(t)), "fitq_rope")
        ctx.save_for_backward(cos_half, sin_half)
        ctx.meta = (heads, dim, seq, rows)
        return out

    @staticmethod
    def backward(ctx, g):
        cos_half, sin_half = ctx.saved_tensors
        heads, dim, seq, rows = ctx.meta
        g = _c(g)
        out = torch.empty_like(g)
        L = _lib.load()
        with torch.cuda.device(g.device):
            _lib.check(L.fitq_rope(g.data_ptr(), out.data_ptr(), cos_half.data_ptr(), sin_half.data_ptr(),
                                   rows, heads, dim, seq, 1, _st(g)), "fitq_rope")
        return out, None, None, None


class SwiGLUFn(torch.autograd.Function):
    """act = silu(gate) * up."""

    @staticmethod
    def forward(ctx, gate, up):
        gate, up = _c(gate), _c(up)
        act = torch.empty_like(gate)
        L = _lib.load()
        with torch.cuda.device(gate.device):
            _lib.check(L.fitq_swiglu_fwd(gate.data_ptr(), up.data_ptr(), act.data_ptr(), gate.numel(),
                                         _st(gate)), "fitq_swiglu_fwd")
        ctx.save_for_backward(gate, up)
        return act

    @staticmethod
    def backward(ctx, d):
        gate, up = ctx.saved_tensors
        d = _c(d.to(gate.dtype))
        dg, du = torch.empty_like(gate), torch.empty_like(up)
        L = _lib.load()
        with torch.cuda.device(gate.device):
            _lib.check(L.fitq_swiglu_bwd(d.data_ptr(), gate.data_ptr(), up.data_ptr(), dg.data_ptr(),
                                         du.data_ptr(), gate.numel(), _st(gate)), "fitq_swiglu_bwd")
        return dg, du


def rms_norm(x, weight, eps):
    return RMSNormFn.apply(x, weight, eps)


def rope(t, cos_half, sin_half, heads):
    return RoPEFn.apply(t, cos_half, sin_half, heads)


def rope_kv_append(q, k, v, cos_half, sin_half, k_cache, v_cache, prefix: int, heads: int,
                   kv_heads: int):
    """Verify step (no autograd): q [B, T, heads*D], k/v [B, T, kv_heads*D]
    bf16 -> rotated q [B, T, heads, D]; rotated k and v written into the
    caches [B, kv_heads, cap, D] at positions [prefix, prefix + T)."""
    b, t = q.shape[0], q.shape[1]
    d = q.shape[-1] // heads
    q, k, v = _c(q), _c(k), _c(v)
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("rope_kv_append: caches must be contiguous")
    out = torch.empty_like(q)
    L = _lib.load()
    with torch.cuda.device(q.device):
        _lib.check(L.fitq_rope_append(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                      k_cache.data_ptr(), v_cache.data_ptr(), _c(cos_half).data_ptr(),
                                      _c(sin_half).data_ptr(), b, t, heads, kv_heads, d, prefix,
                                      int(k_cache.shape[2]), _st(q)), "fitq_rope_append")
    return out.view(b, t, heads, d)


def swiglu_backward(d, gate, up):
    """(d_gate, d_up) of act = silu(gate) * up for upstream d (fitq_swiglu_bwd)."""
    gate, up = _c(gate), _c(up)
    d = _c(d.to(gate.dtype)).view(gate.shape)
    dg, du = torch.empty_like(gate), torch.empty_like(up)
    L = _lib.load()
    with torch.cuda.device(gate.device):
        _lib.check(L.fitq_swiglu_bwd(d.data_ptr(), gate.data_ptr(), up.data_ptr(), dg.data_ptr(),
                                     du.data_ptr(), gate.numel(), _st(gate)), "fitq_swiglu_bwd")
    return dg, du


def swiglu(gate, up):
    return SwiGLUFn.apply(gate, up)


def _check_attention_inputs(q, k, v):
    # the C ABI sees plain pointers: dtype, layout and device are checked here
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError("attention: q, k, v must be [B, S, heads, head_dim]")
    if k.shape != v.shape or k.shape[:2] != q.shape[:2] or k.shape[3] != q.shape[3]:
        raise ValueError(f"attention: q {tuple(q.shape)}, k {tuple(k.shape)}, v {tuple(v.shape)} "
                         "do not match")
    for name, t in (("q", q), ("k", k), ("v", v)):
        if t.dtype != torch.bfloat16 or not t.is_cuda or not t.is_contiguous():
            raise ValueError(f"attention: {name} must be a contiguous bf16 CUDA tensor")
        if t.device != q.device:
            raise ValueError("attention: q, k, v must be on one device")


def attention_forward(q, k, v):
    """Causal GQA attention (fitq_attention_fwd).  q [B, S, H, 128], k/v
    [B, S, KVH, 128] bf16 contiguous; returns (o [B, S, H, 128] bf16, lse
    [B, H, S] fp32, base 2)."""
    _check_attention_inputs(q, k, v)
    b, s, h, d = q.shape
    kvh = k.shape[2]
    o = torch.empty_like(q)
    lse = torch.empty(b, h, s, dtype=torch.float32, device=q.device)
    L = _lib.load()
    with torch.cuda.device(q.device):
        _lib.check(L.fitq_attention_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                        lse.data_ptr(), b, s, h, kvh, d, _st(q)), "fitq_attention_fwd")
    return o, lse


def attention_backward(q, k, v, o, lse, d_o):
    """(dq, dk, dv) of attention_forward for upstream d_o [B, S, H, 128] (fitq_attention_bwd)."""
    _check_attention_inputs(q, k, v)
    if o.shape != q.shape or d_o.shape != q.shape or lse.shape != (q.shape[0], q.shape[2], q.shape[1]):
        raise ValueError("attention_backward: o / d_o must be shaped like q and lse [B, H, S]")
    b, s, h, d = q.shape
    kvh = k.shape[2]
    d_o = _c(d_o.to(q.dtype))
    o, lse = _c(o), _c(lse.float())
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    L = _lib.load()
    with torch.cuda.device(q.device):
        nbytes = L.fitq_attention_bwd_workspace(b, s, h)
        ws = torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=q.device)
        _lib.check(L.fitq_attention_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                        d_o.data_ptr(), lse.data_ptr(), dq.data_ptr(), dk.data_ptr(),
                                        dv.data_ptr(), b, s, h, kvh, d, ws.data_ptr(), nbytes, _st(q)),
                   "fitq_attention_bwd")
    return dq, dk, dv


class AttentionFn(torch.autograd.Function):
    """softmax(q k^T / sqrt(128) + causal mask) v over [B, S, heads, 128]
    tensors, the KV heads shared by heads / kv_heads query heads each."""

    @staticmethod
    def forward(ctx, q, k, v):
        q, k, v = _c(q), _c(k), _c(v)
        o, lse = attention_forward(q, k, v)
        ctx.save_for_backward(q, k, v, o, lse)
        return o

    @staticmethod
    def backward(ctx, d_o):
        q, k, v, o, lse = ctx.saved_tensors
        return attention_backward(q, k, v, o, lse, d_o)


def attention(q, k, v):
    return AttentionFn.apply(q, k, v)
