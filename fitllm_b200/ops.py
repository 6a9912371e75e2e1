"""Functional ops over the C ABI: the QLoRA linear forward/backward, the NF4
GEMV, the raw tcgen05 GEMM and the LoRA optimizer step.  Device tensors in,
device tensors out; every call is asynchronous on the current CUDA stream.
"""
from __future__ import annotations

import ctypes
from typing import List, Optional, Tuple

import torch

from . import _lib
from .nf4 import Nf4WeightCRef, QuantState


def _stream(dev) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _bf16_2d(t: torch.Tensor, cols: int) -> torch.Tensor:
    t = t.reshape(-1, cols)
    if t.dtype != torch.bfloat16:
        t = t.to(torch.bfloat16)
    return t.contiguous()


def _workspace(nbytes: int, dev) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=dev)


def qlora_forward(x2: torch.Tensor, w: Nf4WeightCRef, lora_a: Optional[torch.Tensor],
                  lora_b: Optional[torch.Tensor], scale: float, y_add: Optional[torch.Tensor] = None,
                  want_t: bool = False, gemv: bool = False,
                  bias: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """y[M,N] = x.W^T + scale.(x.A^T).B^T (+ bias) (+ y_add).  x2: bf16 [M, K] contiguous.

    Returns (y, T) with T = x.A^T (bf16 [M, r]) when want_t."""
    L = _lib.load()
    m = x2.shape[0]
    n, k = w.c.n_out, w.c.k_in
    rank = 0 if lora_a is None else int(lora_a.shape[0])
    dev = x2.device
    y = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    t = torch.empty(m, rank, dtype=torch.bfloat16, device=dev) if (want_t and rank) else None
    a = None if lora_a is None else lora_a.detach().to(torch.float32).contiguous()
    b = None if lora_b is None else lora_b.detach().to(torch.float32).contiguous()
    if y_add is not None:
        y_add = _bf16_2d(y_add, n)
    if bias is not None:
        bias = bias.detach().to(torch.bfloat16).contiguous()
    with torch.cuda.device(dev):
        if gemv:
            nbytes = L.fitq_nf4_gemv_workspace(m, n, k, rank)
            ws = _workspace(nbytes, dev)
            _lib.check(L.fitq_nf4_gemv(w.ref, x2.data_ptr(), m, _lib.ptr(a), _lib.ptr(b), rank,
                                       float(scale), _lib.ptr(bias), y.data_ptr(), _lib.ptr(y_add),
                                       ws.data_ptr(),
                                       nbytes, _stream(dev)), "fitq_nf4_gemv")
        else:
            nbytes = L.fitq_qlora_fwd_workspace(m, n, k, rank)
            ws = _workspace(nbytes, dev)
            _lib.check(L.fitq_qlora_fwd(w.ref, x2.data_ptr(), m, _lib.ptr(a), _lib.ptr(b), rank,
                                        float(scale), _lib.ptr(bias), y.data_ptr(), _lib.ptr(y_add),
                                        _lib.ptr(t),
                                        ws.data_ptr(), nbytes, _stream(dev)), "fitq_qlora_fwd")
    return y, t


def qlora_backward(x2: Optional[torch.Tensor], dy2: torch.Tensor, w: Nf4WeightCRef,
                   lora_a: Optional[torch.Tensor], lora_b: Optional[torch.Tensor], scale: float,
                   t_saved: Optional[torch.Tensor] = None, need_dx: bool = True,
                   dx: Optional[torch.Tensor] = None, grad_a: Optional[torch.Tensor] = None,
                   grad_b: Optional[torch.Tensor] = None, grad_accumulate: bool = False):
    """(dx, grad_a, grad_b) of the QLoRA linear for upstream dy2 [M, N] bf16.

    dx: bf16 [M, K] (accumulated into when passed in); grads fp32 in the PEFT
    layouts [r, K] and [N, r] (accumulated into when grad_accumulate)."""
    L = _lib.load()
    m = dy2.shape[0]
    n, k = w.c.n_out, w.c.k_in
    rank = 0 if lora_a is None else int(lora_a.shape[0])
    dev = dy2.device
    dx_acc = dx is not None
    if need_dx and dx is None:
        dx = torch.empty(m, k, dtype=torch.bfloat16, device=dev)
    a = b = None
    if rank:
        a = lora_a.detach().to(torch.float32).contiguous()
        b = lora_b.detach().to(torch.float32).contiguous()
        if grad_a is None:
            grad_a = torch.empty(rank, k, dtype=torch.float32, device=dev)
            grad_b = torch.empty(n, rank, dtype=torch.float32, device=dev)
            grad_accumulate = False
    nbytes = L.fitq_qlora_bwd_workspace(m, n, k, rank)
    ws = _workspace(nbytes, dev)
    with torch.cuda.device(dev):
        _lib.check(L.fitq_qlora_bwd(w.ref, _lib.ptr(x2), dy2.data_ptr(), m, _lib.ptr(a), _lib.ptr(b),
                                    rank, float(scale), _lib.ptr(t_saved),
                                    _lib.ptr(dx) if need_dx else None, int(dx_acc),
                                    _lib.ptr(grad_a), _lib.ptr(grad_b), int(grad_accumulate),
                                    ws.data_ptr(), nbytes, _stream(dev)), "fitq_qlora_bwd")
    return (dx if need_dx else None), grad_a, grad_b


def _gemv_jobs(x2: torch.Tensor, jobs, with_y: bool):
    """The fitq_gemv_job array of (wref, lora_a, lora_b, scale, bias, y_add)
    tuples, the tensors it points at (kept alive by the caller) and, with
    with_y, the bf16 [M, N] outputs it writes."""
    m = x2.shape[0]
    dev = x2.device
    arr = (_lib.GemvJobC * len(jobs))()
    keep, outs = [], []
    for i, (wref, lora_a, lora_b, scale, bias, y_add) in enumerate(jobs):
        n = wref.c.n_out
        y = torch.empty(m, n, dtype=torch.bfloat16, device=dev) if with_y else None
        a = None if lora_a is None else lora_a.detach().to(torch.float32).contiguous()
        b = None if lora_b is None else lora_b.detach().to(torch.float32).contiguous()
        bb = None if bias is None else bias.detach().to(torch.bfloat16).contiguous()
        ya = None if y_add is None else _bf16_2d(y_add, n)
        keep += [a, b, bb, ya]
        arr[i].w = ctypes.pointer(wref.c)
        arr[i].lora_a, arr[i].lora_b = _lib.ptr(a), _lib.ptr(b)
        arr[i].rank = 0 if a is None else int(a.shape[0])
        arr[i].scale = float(scale)
        arr[i].bias, arr[i].y, arr[i].y_add = _lib.ptr(bb), _lib.ptr(y), _lib.ptr(ya)
        outs.append(y)
    return arr, keep, outs


def nf4_gemv_grouped(x2: torch.Tensor, jobs) -> List[torch.Tensor]:
    """Up to three projections of the same x2 [M, K] bf16 in one call
    (fitq_nf4_gemv_grouped).  jobs: (wref, lora_a, lora_b, scale, bias,
    y_add) per projection (None for absent parts).  Returns the bf16 [M, N]
    outputs, each fitq_nf4_gemv's result."""
    L = _lib.load()
    m = x2.shape[0]
    dev = x2.device
    arr, keep, outs = _gemv_jobs(x2, jobs, True)
    with torch.cuda.device(dev):
        nbytes = L.fitq_nf4_gemv_grouped_workspace(arr, len(jobs), m)
        ws = _workspace(nbytes, dev)
        _lib.check(L.fitq_nf4_gemv_grouped(arr, len(jobs), x2.data_ptr(), m, ws.data_ptr(), nbytes,
                                           _stream(dev)), "fitq_nf4_gemv_grouped")
    del keep
    return outs


def nf4_gemv_swiglu(x2: torch.Tensor, gate_job, up_job) -> torch.Tensor:
    """SiLU(x2.Wg^T) * (x2.Wu^T) as bf16 [M, N] (fitq_nf4_gemv_swiglu): the
    gate and up projections (rank 0) and the SwiGLU of their bf16 results."""
    L = _lib.load()
    m = x2.shape[0]
    dev = x2.device
    arr, keep, _ = _gemv_jobs(x2, [gate_job, up_job], False)
    act = torch.empty(m, gate_job[0].c.n_out, dtype=torch.bfloat16, device=dev)
    with torch.cuda.device(dev):
        nbytes = L.fitq_nf4_gemv_swiglu_workspace(arr, m)
        ws = _workspace(nbytes, dev)
        _lib.check(L.fitq_nf4_gemv_swiglu(arr, x2.data_ptr(), m, act.data_ptr(), ws.data_ptr(), nbytes,
                                          _stream(dev)), "fitq_nf4_gemv_swiglu")
    del keep
    return act


def nf4_gateup_swiglu(x2: torch.Tensor, w_gate: Nf4WeightCRef, w_up: Nf4WeightCRef,
                      keep_gate_up: bool = False):
    """act = silu(x.Wg^T) * (x.Wu^T) as ONE tcgen05 GEMM over both NF4 weights
    (fitq_nf4_gateup_swiglu).  x2: bf16 [M, K].  Returns (act, gate, up), bf16
    [M, N]; gate / up only with keep_gate_up (for the backward), else None."""
    L = _lib.load()
    m = x2.shape[0]
    n, k = w_gate.c.n_out, w_gate.c.k_in
    dev = x2.device
    act = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    gate = torch.empty_like(act) if keep_gate_up else None
    up = torch.empty_like(act) if keep_gate_up else None
    with torch.cuda.device(dev):
        nbytes = L.fitq_nf4_gateup_swiglu_workspace(m, n, k)
        ws = _workspace(nbytes, dev)
        _lib.check(L.fitq_nf4_gateup_swiglu(w_gate.ref, w_up.ref, x2.data_ptr(), m, act.data_ptr(),
                                            _lib.ptr(gate), _lib.ptr(up), ws.data_ptr(), nbytes,
                                            _stream(dev)), "fitq_nf4_gateup_swiglu")
    return act, gate, up


def nf4_down_dswiglu(dy2: torch.Tensor, w_down: Nf4WeightCRef, gate: torch.Tensor,
                     up: torch.Tensor):
    """(d_gate, d_up) of act = silu(gate) * up through down_proj: the dX GEMM of
    down_proj with the SwiGLU backward in its epilogue (fitq_nf4_down_dswiglu)."""
    L = _lib.load()
    m = dy2.shape[0]
    k = w_down.c.k_in
    dev = dy2.device
    d_gate = torch.empty(m, k, dtype=torch.bfloat16, device=dev)
    d_up = torch.empty_like(d_gate)
    with torch.cuda.device(dev):
        nbytes = L.fitq_nf4_down_dswiglu_workspace(m, w_down.c.n_out, k)
        ws = _workspace(nbytes, dev)
        _lib.check(L.fitq_nf4_down_dswiglu(w_down.ref, dy2.data_ptr(), m, gate.data_ptr(),
                                           up.data_ptr(), d_gate.data_ptr(), d_up.data_ptr(),
                                           ws.data_ptr(), nbytes, _stream(dev)),
                   "fitq_nf4_down_dswiglu")
    return d_gate, d_up


def verify_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                     prefix: int) -> torch.Tensor:
    """Attention of T new tokens over a KV cache (fitq_verify_attention).

    q: [B, T, H, D] bf16 (post-RoPE); k_cache, v_cache: [B, KVH, cap, D] bf16 with
    the new tokens' keys/values at [prefix, prefix + T).  Returns [B, T, H, D]
    bf16; token i attends to positions <= prefix + i."""
    L = _lib.load()
    b, t, h, d = q.shape
    kvh, cap = int(k_cache.shape[1]), int(k_cache.shape[2])
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("verify_attention: caches must be contiguous [B, KVH, cap, D]")
    q = q.contiguous()
    out = torch.empty_like(q)
    dev = q.device
    with torch.cuda.device(dev):
        nbytes = L.fitq_verify_attention_workspace(b, h, kvh, t, prefix)
        ws = _workspace(nbytes, dev)
        _lib.check(L.fitq_verify_attention(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                                           out.data_ptr(), b, h, kvh, t, prefix, cap, d,
                                           ws.data_ptr(), nbytes, _stream(dev)),
                   "fitq_verify_attention")
    return out


def gemm_bf16_tn(a: torch.Tensor, b: torch.Tensor, c_add: Optional[torch.Tensor] = None) -> torch.Tensor:
    """c = a.b^T (+ c_add) on the tcgen05 tensor cores (bf16 in/out, fp32 accumulate)."""
    L = _lib.load()
    a = a.contiguous()
    b = b.contiguous()
    m, k = a.shape
    n = b.shape[0]
    c = torch.empty(m, n, dtype=torch.bfloat16, device=a.device)
    with torch.cuda.device(a.device):
        _lib.check(L.fitq_gemm_bf16_tn(a.data_ptr(), b.data_ptr(), c.data_ptr(),
                                       _lib.ptr(None if c_add is None else c_add.contiguous()),
                                       m, n, k, _stream(a.device)), "fitq_gemm_bf16_tn")
    return c


def adamw_step(param: torch.Tensor, grad: torch.Tensor, exp_avg: torch.Tensor,
               exp_avg_sq: torch.Tensor, step: int, lr: float, beta1: float, beta2: float,
               eps: float, weight_decay: float, clip: Optional[torch.Tensor] = None) -> None:
    """In-place AdamW on flat fp32 CUDA buffers (fitllm/optimizer.py:206-231 order)."""
    L = _lib.load()
    with torch.cuda.device(param.device):
        _lib.check(L.fitq_adamw_step(param.data_ptr(), grad.data_ptr(), exp_avg.data_ptr(),
                                     exp_avg_sq.data_ptr(), param.numel(), lr, beta1, beta2, eps,
                                     weight_decay, int(step), _lib.ptr(clip),
                                     _stream(param.device)), "fitq_adamw_step")


def grad_clip_coef(flat_grads: torch.Tensor, max_norm: float) -> torch.Tensor:
    """Device fp32 [2] = (global L2 norm, clip coefficient) of a flat fp32 buffer."""
    L = _lib.load()
    out = torch.empty(2, dtype=torch.float32, device=flat_grads.device)
    nbytes = L.fitq_grad_norm_workspace(flat_grads.numel())
    ws = _workspace(nbytes, flat_grads.device)
    with torch.cuda.device(flat_grads.device):
        _lib.check(L.fitq_grad_clip_coef(flat_grads.data_ptr(), flat_grads.numel(), float(max_norm),
                                         out.data_ptr(), ws.data_ptr(), nbytes,
                                         _stream(flat_grads.device)), "fitq_grad_clip_coef")
    return out


def device_status(reset: bool = True) -> int:
    """Synchronise the current stream and return the library's device status word."""
    L = _lib.load()
    return int(L.fitq_get_device_status(int(reset), torch.cuda.current_stream().cuda_stream))
