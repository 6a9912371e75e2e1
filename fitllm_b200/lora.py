"""FitLLM's own LoRA wrapper API (fitllm/lora.py:12-138), B200 edition.

``LoRALinear(base, rank, alpha)`` keeps the reference layout -- ``lora_A``
[in, r] ~ N(0, 0.02), ``lora_B`` [r, out] zeros, ``scale = alpha / rank``,
``forward = base(x) + (x @ A @ B) * scale`` -- and ``LoRAManager`` keeps
``inject_lora`` / ``state_dict`` / ``load_state_dict`` /
``trainable_parameters`` / ``freeze_base_model``.

When the wrapped base is an NF4 ``Linear4bit`` the whole expression runs as
one fused QLoRA call on the sm_100a kernels (the adapter is handed over as the
transposed views A^T [r, in] and B^T [out, r]).  A dense ``nn.Linear`` base
(the reference's unquantised test models) keeps the reference's plain torch
arithmetic, since there is no NF4 weight to stream.
"""
from __future__ import annotations

import logging
from typing import Dict, Iterator, List, Tuple

import torch
import torch.nn as nn

from .qlora import Linear4bit, _QLoRAFunction

logger = logging.getLogger(__name__)


class LoRALinear(nn.Module):
    """forward(x) = base(x) + scale * (x @ A @ B), scale = alpha / rank."""

    def __init__(self, base_linear: nn.Module, rank: int, alpha: float) -> None:
        super().__init__()
        self.base = base_linear
        self.rank = rank
        self.alpha = alpha
        self.scale = alpha / rank
        in_features = base_linear.in_features
        out_features = base_linear.out_features
        dev = next(base_linear.parameters()).device if any(True for _ in base_linear.parameters()) else None
        self.lora_A = nn.Parameter(torch.empty(in_features, rank, device=dev))
        self.lora_B = nn.Parameter(torch.zeros(rank, out_features, device=dev))
        nn.init.normal_(self.lora_A, mean=0.0, std=0.02)
        for p in self.base.parameters():
            p.requires_grad_(False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if isinstance(self.base, Linear4bit):
            if self.rank % 16 == 0 and self.rank <= 64:
                return _QLoRAFunction.apply(x, self.lora_A.t(), self.lora_B.t(), self.base.bias,
                                            self.base.wref(), float(self.scale))
            raise ValueError(f"rank {self.rank}: the NF4 kernels take ranks 16, 32, 48 or 64")
        return self.base(x) + (x @ self.lora_A @ self.lora_B) * self.scale

    def extra_repr(self) -> str:
        return (f"in_features={self.base.in_features}, out_features={self.base.out_features}, "
                f"rank={self.rank}, alpha={self.alpha}")


_LINEAR_TYPES = (nn.Linear, Linear4bit)


class LoRAManager:
    """Injection and persistence of LoRALinear adapters."""

    def __init__(self) -> None:
        self._lora_layers: Dict[str, LoRALinear] = {}

    def inject_lora(self, model: nn.Module, rank: int, alpha: float,
                    targets: Tuple[str, ...] = ("q_proj", "k_proj", "v_proj", "o_proj")) -> nn.Module:
        """Replace every linear (dense or NF4) whose name is, or ends with, a target."""
        self._lora_layers.clear()
        todo: List[Tuple[nn.Module, str, LoRALinear]] = []
        for module_name, module in model.named_modules():
            for child_name, child in module.named_children():
                full = f"{module_name}.{child_name}" if module_name else child_name
                if isinstance(child, _LINEAR_TYPES) and any(
                        child_name == t or full.endswith(t) for t in targets):
                    layer = LoRALinear(child, rank=rank, alpha=alpha)
                    todo.append((module, child_name, layer))
                    self._lora_layers[full] = layer
        for parent, name, layer in todo:
            setattr(parent, name, layer)
        logger.info("Injected LoRA into %d linear layers", len(self._lora_layers))
        return model

    def state_dict(self) -> Dict[str, torch.Tensor]:
        sd: Dict[str, torch.Tensor] = {}
        for name, layer in self._lora_layers.items():
            sd[f"{name}.lora_A"] = layer.lora_A.data.clone()
            sd[f"{name}.lora_B"] = layer.lora_B.data.clone()
        return sd

    def load_state_dict(self, sd: Dict[str, torch.Tensor]) -> None:
        for name, layer in self._lora_layers.items():
            if f"{name}.lora_A" in sd:
                layer.lora_A.data.copy_(sd[f"{name}.lora_A"])
            if f"{name}.lora_B" in sd:
                layer.lora_B.data.copy_(sd[f"{name}.lora_B"])

    def trainable_parameters(self) -> Iterator[nn.Parameter]:
        for layer in self._lora_layers.values():
            yield layer.lora_A
            yield layer.lora_B

    def freeze_base_model(self, model: nn.Module) -> None:
        keep = {id(p) for l in self._lora_layers.values() for p in (l.lora_A, l.lora_B)}
        for p in model.parameters():
            if id(p) not in keep:
                p.requires_grad_(False)

    @property
    def num_lora_layers(self) -> int:
        return len(self._lora_layers)
