"""Drop-in modules for FitLLM's QLoRA projections.

* ``Linear4bit``       -- bitsandbytes ``bnb.nn.Linear4bit`` (NF4, frozen base,
                          optional frozen bias): forward = x.W_nf4^T + bias.
* ``QLoRALinear4bit``  -- PEFT ``lora.Linear4bit`` wrapping a Linear4bit with a
                          rank-r adapter: base(x) + lora_B(lora_A(x)) * scaling,
                          with PEFT's attribute and parameter names
                          (``base_layer``, ``lora_A.default.weight`` [r, K],
                          ``lora_B.default.weight`` [N, r], ``scaling["default"]``).
* ``QLoRAManager``     -- the ``fitllm/qlora.py`` manager API
                          (apply / trainable_parameters / save / load / zero_grad)
                          without a PEFT dependency.

Every forward and backward runs the sm_100a kernels through the C ABI
(``ops.qlora_forward`` / ``ops.qlora_backward``): NF4 dequant fused ahead of a
tcgen05 GEMM whose LoRA term is an extra K-block into the same TMEM
accumulator, or the NF4 GEMV for M <= 64.  CUDA tensors only.
"""
from __future__ import annotations

import json
import math
from pathlib import Path
from typing import Dict, Iterator, List, Optional, Sequence, Tuple

import torch
import torch.nn as nn

from . import ops
from .nf4 import (BLOCKSIZE, Nf4WeightCRef, QuantState, dequantize_nf4, nf4_quant_map,
                  quantize_nf4)

_QS_SUFFIXES = ("absmax", "quant_map", "nested_absmax", "nested_quant_map",
                "quant_state.bitsandbytes__nf4")


class Params4bit(nn.Parameter):
    """Packed NF4 bytes ([N*K/2, 1] uint8, frozen) carrying its QuantState,
    like bitsandbytes' Params4bit."""

    def __new__(cls, data: torch.Tensor, quant_state: Optional[QuantState] = None):
        p = torch.Tensor._make_subclass(cls, data, False)
        p.quant_state = quant_state
        return p


class _QLoRAFunction(torch.autograd.Function):
    """y = x.W^T + s.(x.A^T).B^T (+ bias); grads for x, A and B (W and bias frozen).

    Mirrors bnb MatMul4Bit (dX only through the dequantised weight) plus the
    PEFT LoRA graph (dA, dB), fused into the two C-ABI calls."""

    @staticmethod
    def forward(ctx, x, lora_a, lora_b, bias, wref: Nf4WeightCRef, scale: float, residual=None):
        n, k = wref.c.n_out, wref.c.k_in
        lead = x.shape[:-1]
        x2 = ops._bf16_2d(x, k)
        rank = 0 if lora_a is None else int(lora_a.shape[0])
        # T = x.A^T is kept for dB only when the adapter is trained; the C ABI
        # picks the GEMV kernel for M <= 64 and the tcgen05 GEMM otherwise.
        # A residual is added in the GEMM epilogue (its gradient is dy itself).
        need_t = rank > 0 and (ctx.needs_input_grad[1] or ctx.needs_input_grad[2])
        y, t = ops.qlora_forward(x2, wref, lora_a, lora_b, scale, want_t=need_t, bias=bias,
                                 y_add=residual)
        ctx.res_dtype = None if residual is None else residual.dtype
        ctx.wref = wref
        ctx.scale = scale
        ctx.lead = lead
        ctx.in_dtype = x.dtype
        ctx.rank = rank
        ctx.save_for_backward(x2 if rank else None, lora_a, lora_b, t)
        out = y.view(*lead, n)
        return out if x.dtype == torch.bfloat16 else out.to(x.dtype)

    @staticmethod
    def backward(ctx, dy):
        x2, lora_a, lora_b, t = ctx.saved_tensors
        wref = ctx.wref
        n, k = wref.c.n_out, wref.c.k_in
        dy2 = ops._bf16_2d(dy, n)
        need_dx = ctx.needs_input_grad[0]
        dres = None
        if ctx.res_dtype is not None and ctx.needs_input_grad[6]:
            dres = dy if dy.dtype == ctx.res_dtype else dy.to(ctx.res_dtype)
        if ctx.rank == 0:
            if not need_dx:
                return None, None, None, None, None, None, dres
            dx, _, _ = ops.qlora_backward(None, dy2, wref, None, None, ctx.scale, need_dx=True)
            ga = gb = None
        else:
            dx, ga, gb = ops.qlora_backward(x2, dy2, wref, lora_a, lora_b, ctx.scale, t_saved=t,
                                            need_dx=need_dx)
            ga = ga.to(lora_a.dtype) if ctx.needs_input_grad[1] else None
            gb = gb.to(lora_b.dtype) if ctx.needs_input_grad[2] else None
        if dx is not None:
            dx = dx.view(*ctx.lead, k)
            if ctx.in_dtype != torch.bfloat16:
                dx = dx.to(ctx.in_dtype)
        return dx, ga, gb, None, None, None, dres


def qlora_linear(x: torch.Tensor, weight: Params4bit, lora_a: Optional[torch.Tensor],
                 lora_b: Optional[torch.Tensor], scale: float,
                 bias: Optional[torch.Tensor] = None, wref: Optional[Nf4WeightCRef] = None):
    """Functional QLoRA linear (autograd-aware)."""
    if wref is None:
        wref = Nf4WeightCRef(weight.data, weight.quant_state)
    return _QLoRAFunction.apply(x, lora_a, lora_b, bias, wref, float(scale))


class Linear4bit(nn.Module):
    """NF4 linear layer with frozen weight (and bias), bitsandbytes-compatible
    state-dict keys: ``weight`` plus ``weight.absmax``, ``weight.quant_map``,
    ``weight.nested_absmax``, ``weight.nested_quant_map`` and
    ``weight.quant_state.bitsandbytes__nf4`` (fitllm/forward.py:95-109)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False,
                 compute_dtype: torch.dtype = torch.bfloat16, device=None):
        super().__init__()
        if in_features % BLOCKSIZE:
            raise ValueError(f"in_features={in_features} must be a multiple of {BLOCKSIZE}")
        self.in_features = in_features
        self.out_features = out_features
        self.compute_dtype = compute_dtype
        self.weight = Params4bit(torch.zeros(out_features * in_features // 2, 1, dtype=torch.uint8,
                                             device=device), None)
        if bias:
            self.bias = nn.Parameter(torch.zeros(out_features, dtype=compute_dtype, device=device),
                                     requires_grad=False)
        else:
            self.register_parameter("bias", None)
        self._wref: Optional[Nf4WeightCRef] = None

    # -- construction -----------------------------------------------------
    @classmethod
    def from_float(cls, w: torch.Tensor, bias: Optional[torch.Tensor] = None,
                   compute_dtype: torch.dtype = torch.bfloat16) -> "Linear4bit":
        """Quantise a dense CUDA weight [N, K] with the device NF4 quantiser."""
        n, k = w.shape
        mod = cls(k, n, bias=bias is not None, compute_dtype=compute_dtype, device=w.device)
        packed, qs = quantize_nf4(w, compute_dtype=compute_dtype)
        mod.set_quantized(packed, qs)
        if bias is not None:
            mod.bias.data.copy_(bias.to(compute_dtype))
        return mod

    def set_quantized(self, packed: torch.Tensor, qs: QuantState) -> None:
        self.weight = Params4bit(packed.reshape(-1, 1), qs)
        self._wref = None

    @property
    def quant_state(self) -> Optional[QuantState]:
        return getattr(self.weight, "quant_state", None)

    def wref(self) -> Nf4WeightCRef:
        qs = self.quant_state
        if qs is None:
            raise RuntimeError("Linear4bit has no quant_state: load a quantised shard first")
        w = self._wref
        if w is None or w.c.packed != self.weight.data_ptr() or w.tensors[1] is not qs.absmax:
            w = Nf4WeightCRef(self.weight.data, qs)
            self._wref = w
        return w

    def dequantize(self, dtype=torch.bfloat16) -> torch.Tensor:
        return dequantize_nf4(self.weight.data, self.quant_state, dtype)

    # -- module protocol ----------------------------------------------------
    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        """x.W^T (+ bias) (+ residual, added in the kernel epilogue)."""
        return _QLoRAFunction.apply(x, None, None, self.bias, self.wref(), 1.0, residual)

    def _apply(self, fn, recurse=True):
        qs = self.quant_state
        super()._apply(fn, recurse)
        if qs is not None:
            dev = self.weight.device
            if not isinstance(self.weight, Params4bit):
                self.weight = Params4bit(self.weight.data, None)
            self.weight.quant_state = qs.to(dev) if qs.absmax.device != dev else qs
        self._wref = None
        return self

    def _save_to_state_dict(self, destination, prefix, keep_vars):
        super()._save_to_state_dict(destination, prefix, keep_vars)
        qs = self.quant_state
        if qs is not None:
            for k, v in qs.as_dict(packed=True).items():
                destination[prefix + "weight." + k] = v

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys,
                              unexpected_keys, error_msgs):
        wkey = prefix + "weight"
        qs_dict = {}
        for suf in _QS_SUFFIXES:
            key = wkey + "." + suf
            if key in state_dict:
                qs_dict[suf] = state_dict[key]
        if wkey in state_dict:
            packed = state_dict[wkey]
            dev = self.weight.device
            if qs_dict:
                qs = QuantState.from_dict(qs_dict, device=dev)
            else:
                qs = self.quant_state
            self.weight = Params4bit(packed.to(dev).reshape(-1, 1).contiguous(), qs)
            self._wref = None
        bkey = prefix + "bias"
        if self.bias is not None and bkey in state_dict:
            self.bias.data.copy_(state_dict[bkey].to(self.bias.dtype))
        for key in state_dict:
            if key.startswith(prefix) and key not in (wkey, bkey) and not any(
                    key == wkey + "." + s for s in _QS_SUFFIXES):
                rest = key[len(prefix):]
                if "." not in rest:
                    unexpected_keys.append(key)
        if strict and wkey not in state_dict:
            missing_keys.append(wkey)

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, nf4, bias={self.bias is not None}"


class QLoRALinear4bit(nn.Module):
    """PEFT ``lora.Linear4bit`` equivalent: base Linear4bit + LoRA(r, alpha).

    lora_A.default: nn.Linear(K, r) (Kaiming-uniform a=sqrt(5), PEFT default),
    lora_B.default: nn.Linear(r, N) (zeros), scaling["default"] = alpha / r.
    Dropout is inactive: FitLLM keeps the model in eval() (fitllm/model.py:284)."""

    def __init__(self, base_layer: Linear4bit, r: int = 16, lora_alpha: float = 32.0,
                 lora_dropout: float = 0.0, adapter_name: str = "default"):
        super().__init__()
        if r not in (16, 32, 48, 64):
            raise ValueError(f"rank {r} unsupported (kernels take 16, 32, 48 or 64)")
        self.base_layer = base_layer
        for p in self.base_layer.parameters():
            p.requires_grad_(False)
        self.r = {adapter_name: r}
        self.lora_alpha = {adapter_name: lora_alpha}
        self.scaling = {adapter_name: lora_alpha / r}
        self.lora_dropout_p = lora_dropout
        self.active_adapter = adapter_name
        dev = base_layer.weight.device
        k, n = base_layer.in_features, base_layer.out_features
        self.lora_A = nn.ModuleDict({adapter_name: nn.Linear(k, r, bias=False, device=dev)})
        self.lora_B = nn.ModuleDict({adapter_name: nn.Linear(r, n, bias=False, device=dev)})
        nn.init.kaiming_uniform_(self.lora_A[adapter_name].weight, a=math.sqrt(5))
        nn.init.zeros_(self.lora_B[adapter_name].weight)

    @property
    def in_features(self) -> int:
        return self.base_layer.in_features

    @property
    def out_features(self) -> int:
        return self.base_layer.out_features

    def forward(self, x: torch.Tensor, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        a = self.active_adapter
        return _QLoRAFunction.apply(x, self.lora_A[a].weight, self.lora_B[a].weight,
                                    self.base_layer.bias, self.base_layer.wref(),
                                    float(self.scaling[a]), residual)

    def extra_repr(self) -> str:
        a = self.active_adapter
        return f"r={self.r[a]}, alpha={self.lora_alpha[a]}, scaling={self.scaling[a]}"


def projection_job(mod: nn.Module, y_add: Optional[torch.Tensor] = None):
    """The fitq_gemv_job arguments (wref, lora_a, lora_b, scale, bias, y_add)
    of a Linear4bit or QLoRALinear4bit, for inference."""
    if isinstance(mod, QLoRALinear4bit):
        a = mod.active_adapter
        return (mod.base_layer.wref(), mod.lora_A[a].weight, mod.lora_B[a].weight,
                float(mod.scaling[a]), mod.base_layer.bias, y_add)
    if isinstance(mod, Linear4bit):
        return (mod.wref(), None, None, 1.0, mod.bias, y_add)
    raise TypeError(f"projection_job: not an NF4 projection: {type(mod).__name__}")


@torch.no_grad()
def grouped_forward(mods: Sequence[nn.Module], x: torch.Tensor) -> List[torch.Tensor]:
    """The outputs of up to three projections of the same x in one
    fitq_nf4_gemv_grouped call (no autograd; x.shape[:-1] flattens to M <= 64).
    Same results as calling each module, which the HF layer does one by one
    (fitllm/forward.py:680-686)."""
    lead, k = x.shape[:-1], x.shape[-1]
    ys = ops.nf4_gemv_grouped(ops._bf16_2d(x, k), [projection_job(m) for m in mods])
    return [y.view(*lead, y.shape[-1]) for y in ys]


@torch.no_grad()
def swiglu_forward(gate: nn.Module, up: nn.Module, x: torch.Tensor) -> torch.Tensor:
    """SiLU(gate(x)) * up(x) in one fitq_nf4_gemv_swiglu call (no autograd;
    gate and up without LoRA, M <= 64): the HF MLP's act_fn(gate_proj(x)) *
    up_proj(x) (fitllm/forward.py:680-686), bit-identical to the two modules
    followed by the SwiGLU kernel."""
    lead, k = x.shape[:-1], x.shape[-1]
    act = ops.nf4_gemv_swiglu(ops._bf16_2d(x, k), projection_job(gate), projection_job(up))
    return act.view(*lead, act.shape[-1])


def inject_qlora(model: nn.Module, r: int, alpha: float, targets: Sequence[str]) -> List[str]:
    """Wrap every Linear4bit whose name matches a target suffix (PEFT
    target_modules semantics: exact child name or dotted suffix)."""
    done = []
    for mod_name, mod in list(model.named_modules()):
        for child_name, child in list(mod.named_children()):
            full = f"{mod_name}.{child_name}" if mod_name else child_name
            if isinstance(child, Linear4bit) and any(child_name == t or full.endswith("." + t) or full == t
                                                     for t in targets):
                setattr(mod, child_name, QLoRALinear4bit(child, r=r, lora_alpha=alpha))
                done.append(full)
    return done


class QLoRAManager:
    """fitllm/qlora.py QLoRAManager without PEFT: ``apply`` freezes the model,
    wraps the target Linear4bit modules with rank-r adapters and returns it;
    ``save``/``load`` write/read ``adapter_model.safetensors`` +
    ``adapter_config.json`` with PEFT key names."""

    def __init__(self, rank: int = 16, alpha: float = 32.0,
                 targets: tuple = ("q_proj", "k_proj", "v_proj", "o_proj"),
                 dropout: float = 0.05, bias: str = "none") -> None:
        self.rank = rank
        self.alpha = alpha
        self.targets = list(targets)
        self.dropout = dropout
        self.bias = bias
        self._peft_model: Optional[nn.Module] = None
        self.wrapped: List[str] = []

    def apply(self, model: nn.Module, is_quantized: bool = True) -> nn.Module:
        for p in model.parameters():
            p.requires_grad_(False)
        self.wrapped = inject_qlora(model, self.rank, self.alpha, self.targets)
        self._peft_model = model
        return model

    @property
    def peft_model(self):
        return self._peft_model

    def trainable_parameters(self) -> Iterator[Tuple[str, nn.Parameter]]:
        if self._peft_model is None:
            return
        for name, p in self._peft_model.named_parameters():
            if p.requires_grad:
                yield name, p

    def trainable_param_count(self) -> int:
        return sum(p.numel() for _, p in self.trainable_parameters())

    def adapter_state_dict(self) -> Dict[str, torch.Tensor]:
        """PEFT adapter key names (adapter name dropped, as save_pretrained does)."""
        return {name.replace(".default", ""): p.detach().cpu().contiguous()
                for name, p in self.trainable_parameters()}

    def save(self, path: str) -> None:
        if self._peft_model is None:
            return
        from safetensors.torch import save_file
        out = Path(path)
        out.mkdir(parents=True, exist_ok=True)
        save_file(self.adapter_state_dict(), str(out / "adapter_model.safetensors"))
        (out / "adapter_config.json").write_text(json.dumps({
            "peft_type": "LORA", "r": self.rank, "lora_alpha": self.alpha,
            "target_modules": self.targets, "lora_dropout": self.dropout, "bias": self.bias,
            "task_type": "CAUSAL_LM"}, indent=2))

    def load(self, path: str) -> None:
        if self._peft_model is None:
            raise RuntimeError("QLoRAManager: call apply() before load()")
        from safetensors.torch import load_file
        p = Path(path)
        st = p / "adapter_model.safetensors"
        if not st.exists():
            raise FileNotFoundError(f"No adapter_model.safetensors found in {path}")
        sd = load_file(str(st))
        params = dict(self.trainable_parameters())
        for name, prm in params.items():
            key = name.replace(".default", "")
            if key in sd:
                with torch.no_grad():
                    prm.copy_(sd[key].to(prm.device, prm.dtype))

    def zero_grad(self) -> None:
        for _, p in self.trainable_parameters():
            if p.grad is not None:
                p.grad.zero_()

    def __repr__(self) -> str:
        return (f"QLoRAManager(rank={self.rank}, alpha={self.alpha}, targets={self.targets}, "
                f"trainable_params={self.trainable_param_count():,})")
