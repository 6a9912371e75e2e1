"""Generate the committed golden fixtures under tests/golden/.

    python tests/golden/make_golden.py --reference <FitLLM checkout>

(or with the checkout in the FITLLM_REFERENCE_DIR environment variable)

Two kinds of fixtures:

* reference_torch.pt -- outputs of FitLLM's OWN pure-torch code, imported from
  the reference checkout (which only this script reads; tests and the GPU box
  use the saved file): fitllm.lora.LoRALinear forward/backward on a fixed
  model, fitllm.optimizer.ShardOptimizer.step_from_memory (LoRA mode, three
  steps on a tiny PEFT-named model), fitllm.trainer._clip_lora_accum_grads and
  fitllm.trainer._cosine_lr_scale.
* nf4_vectors.npz -- the CPU oracle's NF4 quantise / dequantise outputs for a
  seeded weight (including an all-zero block and an exact-level block), pinned
  so any change of the restatement is caught.  (No bitsandbytes-produced NF4
  vector is reachable: bitsandbytes is neither vendored nor installed.)
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent


def make_reference_torch(ref_root: str) -> dict:
    sys.path.insert(0, ref_root)
    from fitllm.lora import LoRALinear
    from fitllm.optimizer import ShardOptimizer
    from fitllm.trainer import _clip_lora_accum_grads, _cosine_lr_scale

    out = {}
    # LoRALinear forward/backward (dense fp32 base, reference layout)
    torch.manual_seed(1234)
    base = torch.nn.Linear(32, 48, bias=False)
    lora = LoRALinear(base, rank=16, alpha=32.0)
    with torch.no_grad():
        lora.lora_B.normal_(0.0, 0.05)
    x = torch.randn(2, 5, 32, requires_grad=True)
    y = lora(x)
    gy = torch.randn_like(y)
    y.backward(gy)
    out["lora"] = {"base_w": base.weight.detach().clone(), "A": lora.lora_A.detach().clone(),
                   "B": lora.lora_B.detach().clone(), "x": x.detach().clone(), "gy": gy,
                   "y": y.detach().clone(), "gx": x.grad.clone(), "gA": lora.lora_A.grad.clone(),
                   "gB": lora.lora_B.grad.clone(), "scale": torch.tensor(lora.scale)}

    # ShardOptimizer.step_from_memory (LoRA mode)
    class Peft(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.p = torch.nn.ParameterDict()

    names = ["base_model.model.model.layers.0.self_attn.q_proj.lora_A.default.weight",
             "base_model.model.model.layers.0.self_attn.q_proj.lora_B.default.weight",
             "base_model.model.model.layers.1.self_attn.v_proj.lora_A.default.weight"]

    class Holder(torch.nn.Module):
        def __init__(self):
            super().__init__()
            torch.manual_seed(7)
            self.params = {n: torch.nn.Parameter(torch.randn(4, 6)) for n in names}

        def named_parameters(self, *a, **k):
            return iter(self.params.items())

    model = Holder()
    init = {n: p.detach().clone() for n, p in model.params.items()}
    opt = ShardOptimizer(shard_dir=Path("/tmp/_golden_unused"), num_layers=2, lr=1e-3,
                         weight_decay=0.01, peft_model=model)
    g = torch.Generator().manual_seed(8)
    grads_seq = []
    for step in range(3):
        grads = {0: {"self_attn.q_proj.lora_A.default.weight": torch.randn(4, 6, generator=g),
                     "self_attn.q_proj.lora_B.default.weight": torch.randn(4, 6, generator=g)},
                 1: {"self_attn.v_proj.lora_A.default.weight": torch.randn(4, 6, generator=g)}}
        grads_seq.append({l: {k: v.clone() for k, v in d.items()} for l, d in grads.items()})
        opt.step_from_memory(grads)
    out["adamw"] = {"names": names, "init": init, "grads": grads_seq, "lr": 1e-3, "wd": 0.01,
                    "beta1": 0.9, "beta2": 0.999, "eps": 1e-8,
                    "final": {n: p.detach().clone() for n, p in model.params.items()}}

    # global-norm clip of accumulated grads
    class BE:
        pass

    be = BE()
    g2 = torch.Generator().manual_seed(9)
    be._lora_grad_accum = {0: {"a": torch.randn(100, generator=g2)},
                           1: {"b": torch.randn(50, generator=g2) * 3}}
    before = {l: {k: v.clone() for k, v in d.items()} for l, d in be._lora_grad_accum.items()}
    norm = _clip_lora_accum_grads(be, 1.0)
    out["clip"] = {"before": before, "after": be._lora_grad_accum, "norm": norm, "max_norm": 1.0}
    out["cosine"] = [(s, w, m, _cosine_lr_scale(s, w, m)) for s, w, m in
                     [(0, 10, 100), (5, 10, 100), (10, 10, 100), (55, 10, 100), (100, 10, 100),
                      (150, 10, 100), (3, 0, 7)]]
    return out


def make_nf4_vectors() -> dict:
    sys.path.insert(0, str(ROOT))
    from oracle import nf4 as onf4
    g = torch.Generator().manual_seed(42)
    w = (torch.randn(64, 512, generator=g) * 0.02).numpy().astype(np.float32)
    w[0, :64] = 0.0                                   # all-zero block
    w[1, :64] = onf4.NF4_LEVELS[np.arange(64) % 16] * 0.05  # exact levels x absmax 0.05
    st = onf4.quantize(w)
    return {"w": w, "packed": st.packed, "absmax_code": st.absmax_code,
            "nested_absmax": st.nested_absmax, "offset": np.float32(st.offset),
            "quant_map": st.quant_map, "nested_quant_map": st.nested_quant_map,
            "dequant_bf16": onf4.dequant(st, "bf16"), "dequant_f16": onf4.dequant(st, "f16")}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("FITLLM_REFERENCE_DIR"),
                    help="FitLLM checkout to import (default: $FITLLM_REFERENCE_DIR)")
    a = ap.parse_args()
    if not a.reference:
        ap.error("give --reference or set FITLLM_REFERENCE_DIR")
    torch.save(make_reference_torch(a.reference), HERE / "reference_torch.pt")
    np.savez_compressed(HERE / "nf4_vectors.npz", **make_nf4_vectors())
    print("wrote", HERE / "reference_torch.pt", HERE / "nf4_vectors.npz")


if __name__ == "__main__":
    main()
