"""LoRA parameter store and optimizer step (consumer side of the hot path).

``LoRAStore`` keeps every layer's adapter parameters, gradients and AdamW
moments in four flat fp32 device buffers, one contiguous slice per layer, so

* the per-layer gradient exchange is one NCCL all-reduce over one slice,
* the global-norm clip (_clip_lora_accum_grads, fitllm/trainer.py:70-88) is one
  deterministic device reduction, and
* AdamW (ShardOptimizer.step_from_memory, fitllm/optimizer.py:161-231) is one
  kernel over all parameters, with the reference's update order.

Names follow the PEFT parameter names FitLLM's optimizer matches on
(``...layers.{i}.self_attn.q_proj.lora_A.default.weight``,
fitllm/optimizer.py:183-201).
"""
from __future__ import annotations

import math
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

import torch

from . import ops


def cosine_lr_scale(step: int, warmup_steps: int, max_steps: int) -> float:
    """Linear warmup then cosine decay (fitllm/trainer.py:40-45)."""
    if step < warmup_steps:
        return step / max(1, warmup_steps)
    progress = (step - warmup_steps) / max(1, max_steps - warmup_steps)
    return 0.5 * (1.0 + math.cos(math.pi * min(progress, 1.0)))


class LoRAStore:
    """Flat fp32 param / grad / exp_avg / exp_avg_sq buffers for all layers."""

    def __init__(self, num_layers: int, entries: Sequence[Tuple[str, Tuple[int, ...]]], device):
        """entries: (local name, shape) of one layer's adapter tensors, e.g.
        ("self_attn.q_proj.lora_A.default.weight", (16, 5120))."""
        self.num_layers = num_layers
        self.device = torch.device(device)
        self.local = [(n, tuple(s)) for n, s in entries]
        self.per_layer = sum(math.prod(s) for _, s in self.local)
        total = self.per_layer * num_layers
        self.param = torch.zeros(total, dtype=torch.float32, device=self.device)
        self.grad = torch.zeros_like(self.param)
        self.exp_avg = torch.zeros_like(self.param)
        self.exp_avg_sq = torch.zeros_like(self.param)
        self.step_count = 0

    def layer_slice(self, buf: torch.Tensor, layer: int) -> torch.Tensor:
        return buf[layer * self.per_layer:(layer + 1) * self.per_layer]

    def views(self, buf: torch.Tensor, layer: int) -> Dict[str, torch.Tensor]:
        out, off = {}, layer * self.per_layer
        for name, shape in self.local:
            n = math.prod(shape)
            out[name] = buf[off:off + n].view(shape)
            off += n
        return out

    def full_name(self, layer: int, local: str) -> str:
        return f"base_model.model.model.layers.{layer}.{local}"

    def named_parameters(self) -> Iterable[Tuple[str, torch.Tensor]]:
        for l in range(self.num_layers):
            for name, t in self.views(self.param, l).items():
                yield self.full_name(l, name), t

    def init_layer_(self, layer: int, values: Dict[str, torch.Tensor]) -> None:
        v = self.views(self.param, layer)
        for name, t in values.items():
            v[name].copy_(t.to(v[name].device, torch.float32).view(v[name].shape))

    def bind(self, layer: int, module: torch.nn.Module) -> None:
        """Point the module's adapter parameters (and .grad) at this layer's slices."""
        pv, gv = self.views(self.param, layer), self.views(self.grad, layer)
        for name, p in module.named_parameters():
            if name in pv:
                p.data = pv[name]
                p.grad = gv[name]

    def zero_grad(self) -> None:
        self.grad.zero_()


class ShardOptimizer:
    """AdamW over a LoRAStore, FitLLM's LoRA-mode hyper-parameters and order."""

    def __init__(self, store: LoRAStore, lr: float = 2e-4, weight_decay: float = 0.01,
                 beta1: float = 0.9, beta2: float = 0.999, eps: float = 1e-8,
                 max_grad_norm: float = 1.0):
        self.store = store
        self.lr = lr
        self.weight_decay = weight_decay
        self.beta1 = beta1
        self.beta2 = beta2
        self.eps = eps
        self.max_grad_norm = max_grad_norm
        self.global_step = 0
        self.last_norm: Optional[torch.Tensor] = None

    def set_lr(self, lr: float) -> None:
        self.lr = lr

    def step(self) -> torch.Tensor:
        """Clip (global L2, on device) then AdamW; returns the device [norm, coef] pair."""
        self.global_step += 1
        st = self.store
        clip = ops.grad_clip_coef(st.grad, self.max_grad_norm)
        ops.adamw_step(st.param, st.grad, st.exp_avg, st.exp_avg_sq, self.global_step, self.lr,
                       self.beta1, self.beta2, self.eps, self.weight_decay, clip=clip)
        self.last_norm = clip
        return clip

    def step_from_memory(self, grad_accum: Dict[int, Dict[str, torch.Tensor]]) -> None:
        """Reference-shaped entry: {layer_idx: {param_name: grad}} -> one AdamW step
        (grads are copied into the store; names are matched by suffix like
        fitllm/optimizer.py:183-201)."""
        st = self.store
        gviews = {l: st.views(st.grad, l) for l in range(st.num_layers)}
        st.zero_grad()
        for layer, grads in grad_accum.items():
            for name, g in grads.items():
                hit = [k for k in gviews[layer] if name.endswith(k) or k.endswith(name)]
                if hit:
                    gviews[layer][hit[0]].copy_(g.to(st.device, torch.float32).view(gviews[layer][hit[0]].shape))
        self.step()
