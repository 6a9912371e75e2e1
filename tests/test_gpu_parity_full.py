"""GPU parity at the benchmarked shapes.

The other kernel tests use shapes where every CTA gets one tile.  These run
the shapes the benchmarks run, so the persistent multi-tile loop, the
double-buffered TMEM accumulator (epilogue of tile i overlapping the main
loop of tile i+1) and several raster groups all execute under a check:

* the single q_proj QLoRA linear of the CPU-runnable workload at full size
  (x [512, 5120], W 5120x5120 NF4, r=16, alpha=32; seeds 0-4 for W, A, B, x,
  dY) against the fp64 oracle, forward and backward, on every GEMM path
  (dequant + either bf16 GEMM kernel, NF4 decoded inside the GEMM);
* the tcgen05 GEMM at shapes with >= 3 tiles per CTA and >= 2 raster groups
  (on the pair kernel also the wide-N raster branch), including one K >= 4N
  shape, against an fp32 torch product;
* QLoRA forward / backward at training token counts of one micro-batch pair
  (M = 4096) on q_proj and down_proj shapes, against fp32 torch on the
  oracle's dequantised weights;
* one full Qwen2.5-32B-shaped decoder layer (hidden 5120, 40/8 heads of 128,
  intermediate 27648, LoRA r=16 on q/v) on one 1 x 512 micro-batch, forward
  and backward, against the fp32 CPU restatement of the layer.

Tolerance: 1e-2 relative Frobenius norm for outputs and gradients (bf16
operands, fp32 accumulation); 4e-3 for the plain bf16 GEMM.
"""
import json
import math

import numpy as np
import pytest
import torch

from oracle import layer_ref
from oracle import nf4 as onf4

pytestmark = pytest.mark.gpu
REL = 1e-2
GEMM_REL = 4e-3


PATHS = ["dequant+1cta", "dequant+2cta", "fused", "auto"]


def _set_path(monkeypatch, path):
    """Select the GEMM path: NF4 materialised then a bf16 GEMM on either
    tcgen05 kernel, NF4 decoded inside the GEMM, or the library's choice."""
    if path.startswith("dequant"):
        monkeypatch.setenv("FITQ_NF4_FUSED", "0")
        monkeypatch.setenv("FITQ_GEMM_VARIANT", path.split("+")[1])
    elif path == "fused":
        monkeypatch.setenv("FITQ_NF4_FUSED", "1")


def _state_to_device(st, dev):
    from fitllm_b200.nf4 import Nf4WeightCRef, QuantState
    packed = torch.from_numpy(st.packed.copy()).to(dev)
    qs = QuantState(absmax=torch.from_numpy(st.absmax_code.copy()).to(dev), shape=st.shape,
                    quant_map=torch.from_numpy(st.quant_map.copy()).to(dev),
                    nested_absmax=torch.from_numpy(st.nested_absmax.copy()).to(dev),
                    nested_quant_map=torch.from_numpy(st.nested_quant_map.copy()).to(dev),
                    offset=float(st.offset))
    return Nf4WeightCRef(packed, qs)


@pytest.fixture(scope="module")
def qproj_case():
    """The single-linear workload: seeds 0 (W), 1 (A), 2 (B), 3 (x), 4 (dY)."""
    n = k = 5120
    m, r = 512, 16
    w = (torch.randn(n, k, generator=torch.Generator().manual_seed(0)) * 0.02).numpy()
    st = onf4.quantize(w)
    w_deq = onf4.bf16_bits_to_f32(onf4.dequant(st, "bf16"))
    bound = 1.0 / math.sqrt(k)  # kaiming_uniform(a=sqrt(5)) on a [r, K] weight
    A = (torch.rand(r, k, generator=torch.Generator().manual_seed(1)) * 2 - 1) * bound
    B = torch.randn(n, r, generator=torch.Generator().manual_seed(2)) * 0.01
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(3)).bfloat16()
    dy = torch.randn(m, n, generator=torch.Generator().manual_seed(4)).bfloat16()
    s = 32.0 / r
    y_ref = onf4.qlora_forward(x.float().numpy(), w_deq, A.numpy(), B.numpy(), s)
    grads = onf4.qlora_backward(x.float().numpy(), w_deq, A.numpy(), B.numpy(), s, dy.float().numpy())
    return dict(st=st, A=A, B=B, x=x, dy=dy, s=s, y_ref=y_ref, grads=grads)


@pytest.mark.parametrize("path", PATHS)
def test_qproj_linear_full_shape_vs_oracle(cuda_dev, qproj_case, path, monkeypatch):
    """Config-1 shape (512 x 5120 x 5120, r=16) through ops.qlora_forward /
    qlora_backward: y, dX, dA, dB within 1e-2 of the fp64 oracle."""
    _set_path(monkeypatch, path)
    from fitllm_b200 import ops
    c = qproj_case
    wref = _state_to_device(c["st"], cuda_dev)
    xd, dyd = c["x"].to(cuda_dev), c["dy"].to(cuda_dev)
    Ad, Bd = c["A"].to(cuda_dev), c["B"].to(cuda_dev)
    y, t = ops.qlora_forward(xd, wref, Ad, Bd, c["s"], want_t=True)
    assert onf4.rel_err(y.float().cpu().numpy(), c["y_ref"]) < REL
    dx, ga, gb = ops.qlora_backward(xd, dyd, wref, Ad, Bd, c["s"], t_saved=t)
    rdx, rda, rdb = c["grads"]
    assert onf4.rel_err(dx.float().cpu().numpy(), rdx) < REL
    assert onf4.rel_err(ga.cpu().numpy(), rda) < REL
    assert onf4.rel_err(gb.cpu().numpy(), rdb) < REL
    assert ops.device_status() == 0


# (M, N, K): 1-CTA tiles per CTA / raster groups; pair tiles per pair / groups
#   8192 x 5120 x 1024: 1280 tiles (8.6 per CTA), 4 groups; 640 pair tiles, wide-N groups
#   4096 x 4096 x 5120: 512 tiles (3.5 per CTA), 2 groups; 256 pair tiles, wide-N groups
#   4096 x 1024 x 5120: K >= 4N (the one-CTA dispatch), 128 tiles; 64 pair tiles
#   2048 x 27648 x 5120: gate_proj of one 2048-token micro-batch, 1728 tiles
@pytest.mark.parametrize("m,n,k", [(8192, 5120, 1024), (4096, 4096, 5120), (4096, 1024, 5120),
                                   (2048, 27648, 5120)])
@pytest.mark.parametrize("variant", ["1cta", "2cta"])
def test_gemm_multi_tile_raster(cuda_dev, m, n, k, variant, monkeypatch):
    """Persistent tile loop, double-buffered accumulators and several raster
    groups of both tcgen05 GEMMs against fp32 torch, with and without the
    residual add of the epilogue."""
    monkeypatch.setenv("FITQ_GEMM_VARIANT", variant)
    from fitllm_b200 import ops
    torch.backends.cuda.matmul.allow_tf32 = False
    g = torch.Generator(device=cuda_dev).manual_seed(m + n + k)
    a = torch.randn(m, k, generator=g, device=cuda_dev).bfloat16()
    b = torch.randn(n, k, generator=g, device=cuda_dev).bfloat16()
    add = torch.randn(m, n, generator=g, device=cuda_dev).bfloat16()
    ref = a.float() @ b.float().T
    c = ops.gemm_bf16_tn(a, b)
    assert float((c.float() - ref).norm() / ref.norm()) < GEMM_REL
    c2 = ops.gemm_bf16_tn(a, b, add)
    ref2 = ref + add.float()
    assert float((c2.float() - ref2).norm() / ref2.norm()) < GEMM_REL
    # every tile written: no row block or column block left at its initial value
    blocks = (c.float() - ref).abs().view(m // 128, 128, n // 64, 64).amax(dim=(1, 3))
    assert float(blocks.max()) < 0.05 * float(ref.abs().max())
    assert ops.device_status() == 0


def _torch_qlora_ref(x, w, A, B, s, dy):
    """fp32 torch restatement of the QLoRA linear: y, dX, dA, dB."""
    xf, wf, Af, Bf, dyf = (t.float() for t in (x, w, A, B, dy))
    y = xf @ wf.T + s * (xf @ Af.T) @ Bf.T
    T = xf @ Af.T
    U = dyf @ Bf
    return y, dyf @ wf + s * U @ Af, s * U.T @ xf, s * dyf.T @ T


@pytest.mark.parametrize("m,n,k", [(4096, 5120, 5120), (2048, 5120, 27648), (4096, 1024, 5120)])
@pytest.mark.parametrize("path", PATHS)
def test_qlora_training_shapes_vs_torch(cuda_dev, m, n, k, path, monkeypatch):
    """QLoRA forward + backward at training token counts (q_proj, down_proj,
    v_proj shapes) against fp32 torch on the oracle-dequantised weights."""
    _set_path(monkeypatch, path)
    from fitllm_b200 import ops
    torch.backends.cuda.matmul.allow_tf32 = False
    r, s = 16, 2.0
    gw = torch.Generator().manual_seed(n + k)
    st = onf4.quantize((torch.randn(n, k, generator=gw) * 0.02).numpy())
    wref = _state_to_device(st, cuda_dev)
    w = torch.from_numpy(onf4.bf16_bits_to_f32(onf4.dequant(st, "bf16"))).to(cuda_dev)
    g = torch.Generator(device=cuda_dev).manual_seed(m + 3)
    A = (torch.rand(r, k, generator=g, device=cuda_dev) * 2 - 1) / math.sqrt(k)
    B = torch.randn(n, r, generator=g, device=cuda_dev) * 0.01
    x = torch.randn(m, k, generator=g, device=cuda_dev).bfloat16()
    dy = torch.randn(m, n, generator=g, device=cuda_dev).bfloat16()
    y, t = ops.qlora_forward(x, wref, A, B, s, want_t=True)
    dx, ga, gb = ops.qlora_backward(x, dy, wref, A, B, s, t_saved=t)
    ry, rdx, rda, rdb = _torch_qlora_ref(x, w, A, B, s, dy)
    for got, ref in ((y, ry), (dx, rdx), (ga, rda), (gb, rdb)):
        assert float((got.float() - ref).norm() / ref.norm()) < REL
    assert ops.device_status() == 0


FULL = dict(hidden=5120, heads=40, kv_heads=8, head_dim=128, inter=27648)
_HF_PARENT = {"q_proj": "self_attn", "k_proj": "self_attn", "v_proj": "self_attn",
              "o_proj": "self_attn", "gate_proj": "mlp", "up_proj": "mlp", "down_proj": "mlp"}


def _full_layer_shard(seed):
    """Flat bitsandbytes shard keys (fitllm/forward.py:95-109 layout) of one
    Qwen2.5-32B-shaped layer quantised by the C oracle, and the oracle's
    weight dict (dequantised fp32 weights, biases, LoRA A/B)."""
    g = torch.Generator().manual_seed(seed)
    shard, ref = {}, {}
    for name, kind, bias in layer_ref.PROJ:
        n, k = layer_ref.proj_shape(kind, FULL["hidden"], FULL["heads"], FULL["kv_heads"],
                                    FULL["head_dim"], FULL["inter"])
        st = onf4.quantize((torch.randn(n, k, generator=g) * 0.02).numpy())
        key = f"{_HF_PARENT[name]}.{name}.weight"
        shard[key] = torch.from_numpy(st.packed).view(-1, 1)
        shard[key + ".absmax"] = torch.from_numpy(st.absmax_code)
        shard[key + ".quant_map"] = torch.from_numpy(st.quant_map)
        shard[key + ".nested_absmax"] = torch.from_numpy(st.nested_absmax)
        shard[key + ".nested_quant_map"] = torch.from_numpy(st.nested_quant_map)
        meta = {"quant_type": "nf4", "blocksize": 64, "dtype": "bfloat16", "shape": [n, k],
                "nested_blocksize": 256, "nested_dtype": "float32", "nested_offset": float(st.offset)}
        shard[key + ".quant_state.bitsandbytes__nf4"] = torch.tensor(
            list(json.dumps(meta).encode()), dtype=torch.uint8)
        ref[name] = torch.from_numpy(onf4.bf16_bits_to_f32(onf4.dequant(st, "bf16")))
        if bias:
            b = (torch.randn(n, generator=g) * 0.02).bfloat16()
            shard[f"{_HF_PARENT[name]}.{name}.bias"] = b
            ref[name + ".bias"] = b.float()
    shard["input_layernorm.weight"] = torch.ones(FULL["hidden"], dtype=torch.bfloat16)
    shard["post_attention_layernorm.weight"] = torch.ones(FULL["hidden"], dtype=torch.bfloat16)
    for name in ("q_proj", "v_proj"):
        n, k = ref[name].shape
        ref[name + ".lora_A"] = (torch.rand(16, k, generator=g) * 2 - 1) / math.sqrt(k)
        ref[name + ".lora_B"] = torch.randn(n, 16, generator=g) * 0.01
    ref["scale"] = torch.tensor(2.0)
    ref["cfg"] = torch.tensor([FULL["hidden"], FULL["heads"], FULL["kv_heads"], FULL["head_dim"],
                               FULL["inter"]])
    return shard, ref


def _restated_layer(ref, h, go, dtype, device):
    """Output, input gradient and LoRA gradients of the restated layer in
    `dtype` on `device` (fp32 host: the oracle; bf16 GPU: the reference's own
    precision -- bf16 activations, fp32-accumulating matmuls)."""
    ww = {k: (v if k in ("scale", "cfg") else v.to(device, dtype)) for k, v in ref.items()}
    params = {k: ww[k].clone().requires_grad_(True) for k in ww if "lora_" in k}
    ww.update(params)
    x = h.to(device, dtype).clone().requires_grad_(True)
    y = layer_ref.layer_forward(ww, x)
    y.backward(go.to(device, dtype))
    out = {"y": y.detach().float().cpu(), "dx": x.grad.float().cpu()}
    out.update({k: p.grad.float().cpu() for k, p in params.items()})
    return out


def test_full_qwen25_32b_layer_vs_restatement(cuda_dev):
    """One Qwen2.5-32B-shaped decoder layer, 1 x 512 tokens: output, input
    gradient and the q/v LoRA gradients against the fp32 CPU restatement.

    The bound is 1e-2 relative, or the error of the reference's own precision
    regime where that is larger: the same layer restated in bf16 (what
    FitLLM's autocast path computes) is 1.2e-2 (output) to 1.8e-2 (LoRA
    gradients) from fp32 at this size, so a bf16 implementation cannot be
    held below it; this one must be at least as close to fp32 as that."""
    from fitllm_b200.layer import DecoderLayer, LayerConfig, add_lora_
    cfg = LayerConfig(lora_rank=16, lora_alpha=32.0, lora_targets=("q_proj", "v_proj"))
    shard, ref = _full_layer_shard(71)
    layer = DecoderLayer(cfg, device=cuda_dev)
    layer.load_state_dict(shard, strict=False)
    add_lora_(layer, 16, 32.0, ("q_proj", "v_proj"), seed=0)
    with torch.no_grad():
        for name in ("q_proj", "v_proj"):
            mod = layer.self_attn.get_submodule(name)
            mod.lora_A["default"].weight.copy_(ref[name + ".lora_A"])
            mod.lora_B["default"].weight.copy_(ref[name + ".lora_B"])
    del shard
    g = torch.Generator().manual_seed(72)
    h = torch.randn(1, 512, FULL["hidden"], generator=g).bfloat16()
    go = torch.randn(1, 512, FULL["hidden"], generator=g).bfloat16()
    hd = h.to(cuda_dev).requires_grad_(True)
    y = layer(hd)
    y.backward(go.to(cuda_dev))
    torch.cuda.synchronize()
    mine = {"y": y.detach().float().cpu(), "dx": hd.grad.float().cpu()}
    for name in ("q_proj", "v_proj"):
        mod = layer.self_attn.get_submodule(name)
        mine[name + ".lora_A"] = mod.lora_A["default"].weight.grad.float().cpu()
        mine[name + ".lora_B"] = mod.lora_B["default"].weight.grad.float().cpu()
    r32 = _restated_layer(ref, h, go, torch.float32, "cpu")
    r16 = _restated_layer(ref, h, go, torch.bfloat16, cuda_dev)
    for key, got in mine.items():
        err = onf4.rel_err(got.numpy(), r32[key].numpy())
        err_bf16 = onf4.rel_err(r16[key].numpy(), r32[key].numpy())
        assert err < max(REL, err_bf16), (key, err, err_bf16)
    assert onf4.rel_err(mine["y"].numpy(), r32["y"].numpy()) < REL
