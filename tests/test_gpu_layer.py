"""GPU parity of the module API, the decoder layer and the shard-stationary
engine against the CPU restatement (oracle/layer_ref.py), on small shapes.

Weights are quantised by the C oracle on the host and loaded through the
bitsandbytes flat shard keys (fitllm/forward.py:95-109 layout), so these tests
also cover QuantState (de)serialisation and the scheduler's pinned ring.
Tolerance: 1e-2 relative Frobenius norm (bf16 operands, fp32 accumulation),
the north-star contract for outputs and gradients.
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

SMALL = dict(hidden=256, heads=4, kv_heads=2, head_dim=64, inter=512)


def _cfg():
    from fitllm_b200.layer import LayerConfig
    return LayerConfig(hidden=SMALL["hidden"], heads=SMALL["heads"], kv_heads=SMALL["kv_heads"],
                       head_dim=SMALL["head_dim"], intermediate=SMALL["inter"], lora_rank=16,
                       lora_alpha=32.0, lora_targets=("q_proj", "v_proj"))


def _oracle_shard(seed):
    """(flat shard dict for my layer, oracle weight dict) built from one seed."""
    g = torch.Generator().manual_seed(seed)
    shard, ref = {}, {}
    names = {"q_proj": "self_attn", "k_proj": "self_attn", "v_proj": "self_attn",
             "o_proj": "self_attn", "gate_proj": "mlp", "up_proj": "mlp", "down_proj": "mlp"}
    for name, kind, bias in layer_ref.PROJ:
        n, k = layer_ref.proj_shape(kind, SMALL["hidden"], SMALL["heads"], SMALL["kv_heads"],
                                    SMALL["head_dim"], SMALL["inter"])
        st = onf4.quantize((torch.randn(n, k, generator=g) * 0.02).numpy())
        key = f"{names[name]}.{name}.weight"
        shard[key] = torch.from_numpy(st.packed.copy()).view(-1, 1)
        shard[key + ".absmax"] = torch.from_numpy(st.absmax_code.copy())
        shard[key + ".quant_map"] = torch.from_numpy(st.quant_map.copy())
        shard[key + ".nested_absmax"] = torch.from_numpy(st.nested_absmax.copy())
        shard[key + ".nested_quant_map"] = torch.from_numpy(st.nested_quant_map.copy())
        meta = {"quant_type": "nf4", "blocksize": 64, "dtype": "bfloat16", "shape": [n, k],
                "nested_blocksize": 256, "nested_dtype": "float32", "nested_offset": float(st.offset)}
        shard[key + ".quant_state.bitsandbytes__nf4"] = torch.tensor(
            list(json.dumps(meta).encode()), dtype=torch.uint8)
        ref[name] = torch.from_numpy(onf4.bf16_bits_to_f32(onf4.dequant(st, "bf16")))
        if bias:
            b = (torch.randn(n, generator=g) * 0.02).bfloat16()
            shard[f"{names[name]}.{name}.bias"] = b
            ref[name + ".bias"] = b.float()
    shard["input_layernorm.weight"] = torch.ones(SMALL["hidden"], dtype=torch.bfloat16)
    shard["post_attention_layernorm.weight"] = torch.ones(SMALL["hidden"], dtype=torch.bfloat16)
    for name in ("q_proj", "v_proj"):
        n, k = ref[name].shape
        ref[name + ".lora_A"] = (torch.rand(16, k, generator=g) * 2 - 1) / math.sqrt(k)
        ref[name + ".lora_B"] = torch.randn(n, 16, generator=g) * 0.02
    ref["scale"] = torch.tensor(2.0)
    ref["cfg"] = torch.tensor([SMALL["hidden"], SMALL["heads"], SMALL["kv_heads"],
                               SMALL["head_dim"], SMALL["inter"]])
    return shard, ref


def _layer_from_shard(shard, ref, dev):
    from fitllm_b200.layer import DecoderLayer, add_lora_
    layer = DecoderLayer(_cfg(), device=dev)
    missing, unexpected = layer.load_state_dict({k: v for k, v in shard.items()}, strict=False)
    add_lora_(layer, 16, 32.0, ("q_proj", "v_proj"), seed=0)
    with torch.no_grad():
        for name in ("q_proj", "v_proj"):
            mod = layer.self_attn.get_submodule(name)
            mod.lora_A["default"].weight.copy_(ref[name + ".lora_A"])
            mod.lora_B["default"].weight.copy_(ref[name + ".lora_B"])
    return layer


def test_qlora_linear_module_autograd(cuda_dev):
    from fitllm_b200.qlora import Linear4bit, QLoRALinear4bit, QLoRAManager
    n, k, m = 384, 512, 200
    g = torch.Generator().manual_seed(3)
    st = onf4.quantize((torch.randn(n, k, generator=g) * 0.02).numpy())
    w = onf4.bf16_bits_to_f32(onf4.dequant(st, "bf16"))
    lin = Linear4bit(k, n, bias=True, device=cuda_dev)
    sd = {"weight": torch.from_numpy(st.packed.copy()).view(-1, 1),
          "weight.absmax": torch.from_numpy(st.absmax_code.copy()),
          "weight.quant_map": torch.from_numpy(st.quant_map.copy()),
          "weight.nested_absmax": torch.from_numpy(st.nested_absmax.copy()),
          "weight.nested_quant_map": torch.from_numpy(st.nested_quant_map.copy()),
          "weight.quant_state.bitsandbytes__nf4": torch.tensor(list(json.dumps(
              {"quant_type": "nf4", "blocksize": 64, "dtype": "bfloat16", "shape": [n, k],
               "nested_blocksize": 256, "nested_dtype": "float32",
               "nested_offset": float(st.offset)}).encode()), dtype=torch.uint8),
          "bias": (torch.randn(n, generator=g) * 0.1).bfloat16()}
    lin.load_state_dict(sd)
    # dequantised values through the module are the oracle's bits
    assert np.array_equal(lin.dequantize().view(torch.int16).cpu().numpy().view(np.uint16),
                          onf4.dequant(st, "bf16"))
    # state_dict round trip keeps the flat key set
    sd2 = lin.state_dict()
    assert set(sd2) == set(sd)
    q = QLoRALinear4bit(lin, r=16, lora_alpha=32.0)
    with torch.no_grad():
        q.lora_B["default"].weight.normal_(0, 0.02)
    x = torch.randn(m, k, generator=g).bfloat16().to(cuda_dev).requires_grad_(True)
    y = q(x)
    dy = torch.randn(m, n, generator=g).bfloat16().to(cuda_dev)
    y.backward(dy)
    A = q.lora_A["default"].weight.detach().cpu().numpy()
    B = q.lora_B["default"].weight.detach().cpu().numpy()
    bias = sd["bias"].float().numpy()
    ry = onf4.qlora_forward(x.detach().float().cpu().numpy(), w, A, B, 2.0) + bias
    assert onf4.rel_err(y.detach().float().cpu().numpy(), ry) < REL
    rdx, rda, rdb = onf4.qlora_backward(x.detach().float().cpu().numpy(), w, A, B, 2.0,
                                        dy.float().cpu().numpy())
    assert onf4.rel_err(x.grad.float().cpu().numpy(), rdx) < REL
    assert onf4.rel_err(q.lora_A["default"].weight.grad.cpu().numpy(), rda) < REL
    assert onf4.rel_err(q.lora_B["default"].weight.grad.cpu().numpy(), rdb) < REL
    assert lin.weight.grad is None and lin.bias.grad is None
    mgr = QLoRAManager(rank=16, alpha=32.0, targets=("q_proj",))
    assert "lora_A.default.weight" in dict(q.named_parameters())


def test_lora_linear_own_layout_on_nf4(cuda_dev):
    """fitllm/lora.py layout (A [in, r], B [r, out]) over an NF4 base."""
    from fitllm_b200.lora import LoRALinear
    from fitllm_b200.qlora import Linear4bit
    n, k, m = 256, 256, 96
    g = torch.Generator(device=cuda_dev).manual_seed(1)
    base = Linear4bit.from_float(torch.randn(n, k, generator=g, device=cuda_dev) * 0.02)
    lora = LoRALinear(base, rank=16, alpha=32.0)
    with torch.no_grad():
        lora.lora_B.normal_(0, 0.02)
    x = torch.randn(m, k, device=cuda_dev).bfloat16().requires_grad_(True)
    y = lora(x)
    w = base.dequantize().float()
    ref = x.detach().float() @ w.T + 2.0 * (x.detach().float() @ lora.lora_A.detach()) @ lora.lora_B.detach()
    assert onf4.rel_err(y.detach().float().cpu().numpy(), ref.cpu().numpy()) < REL
    y.float().sum().backward()
    assert lora.lora_A.grad is not None and lora.lora_B.grad is not None
    assert lora.lora_A.grad.shape == (k, 16) and lora.lora_B.grad.shape == (16, n)


def test_decoder_layer_vs_restatement(cuda_dev):
    shard, ref = _oracle_shard(11)
    layer = _layer_from_shard(shard, ref, cuda_dev)
    g = torch.Generator().manual_seed(12)
    h = torch.randn(2, 128, SMALL["hidden"], generator=g).bfloat16()
    go = torch.randn(2, 128, SMALL["hidden"], generator=g).bfloat16()
    hd = h.to(cuda_dev).requires_grad_(True)
    y = layer(hd)
    y.backward(go.to(cuda_dev))
    rgx, rg = layer_ref.layer_step(ref, h.float(), go.float())
    ry = layer_ref.layer_forward(ref, h.float())
    assert onf4.rel_err(y.detach().float().cpu().numpy(), ry.detach().numpy()) < REL
    assert onf4.rel_err(hd.grad.float().cpu().numpy(), rgx.numpy()) < REL
    for name in ("q_proj", "v_proj"):
        mod = layer.self_attn.get_submodule(name)
        assert onf4.rel_err(mod.lora_A["default"].weight.grad.cpu().numpy(),
                            rg[name + ".lora_A"].numpy()) < REL
        assert onf4.rel_err(mod.lora_B["default"].weight.grad.cpu().numpy(),
                            rg[name + ".lora_B"].numpy()) < REL


@pytest.mark.parametrize("mb_chunk,keep", [(1, 0), (None, 2), (None, 1)])
def test_engine_two_layers_vs_restatement(cuda_dev, mb_chunk, keep):
    """Shard-stationary forward + backward over 2 layers streamed through the
    pinned host ring, LoRA grads accumulated in the flat store; with the
    recompute (keep=0), without it (keep=2) and mixed (keep=1)."""
    from fitllm_b200.engine import ShardStationaryEngine, lora_entries
    from fitllm_b200.layer import DecoderLayer, add_lora_
    from fitllm_b200.optimizer import LoRAStore
    from fitllm_b200.scheduler import ShardScheduler
    cfg = _cfg()
    shards, refs = [], []
    for l in range(2):
        s, r = _oracle_shard(20 + l)
        shards.append(s)
        refs.append(r)
    sched = ShardScheduler(2, cuda_dev, ring_slots=2)
    for l in range(2):
        sched.add_layer(l, shards[l])
    proto = DecoderLayer(cfg, device=cuda_dev)
    add_lora_(proto, 16, 32.0, cfg.lora_targets, seed=0)
    store = LoRAStore(2, lora_entries(proto), cuda_dev)
    for l in range(2):
        store.init_layer_(l, {f"self_attn.{n}.lora_{ab}.default.weight": refs[l][f"{n}.lora_{ab}"]
                              for n in ("q_proj", "v_proj") for ab in ("A", "B")})
    eng = ShardStationaryEngine(cfg, sched, store, cuda_dev, mb_chunk=mb_chunk, keep_activations=keep)
    g = torch.Generator().manual_seed(30)
    h = torch.randn(3, 64, SMALL["hidden"], generator=g).bfloat16()
    go = torch.randn(3, 64, SMALL["hidden"], generator=g).bfloat16()
    store.zero_grad()
    acts = eng.forward(h.to(cuda_dev))
    gin = eng.backward(acts, go.to(cuda_dev))
    # CPU restatement with autograd through both layers
    params = {l: {k: refs[l][k].clone().requires_grad_(True) for k in refs[l] if "lora_" in k}
              for l in range(2)}
    x = h.float().clone().requires_grad_(True)
    y = x
    for l in range(2):
        ww = dict(refs[l])
        ww.update(params[l])
        y = layer_ref.layer_forward(ww, y)
    y.backward(go.float())
    assert onf4.rel_err(acts[2].float().cpu().numpy(), y.detach().numpy()) < REL
    assert onf4.rel_err(gin.float().cpu().numpy(), x.grad.numpy()) < REL
    for l in range(2):
        gv = store.views(store.grad, l)
        for n in ("q_proj", "v_proj"):
            for ab in ("A", "B"):
                got = gv[f"self_attn.{n}.lora_{ab}.default.weight"].cpu().numpy()
                assert onf4.rel_err(got, params[l][f"{n}.lora_{ab}"].grad.numpy()) < REL


def test_optimizer_step_matches_reference_math(cuda_dev):
    """Device AdamW + clip vs the reference update order restated in fp32 torch."""
    from fitllm_b200 import ops
    g = torch.Generator().manual_seed(2)
    p = torch.randn(10000, generator=g)
    grads = [torch.randn(10000, generator=g) * 0.3 for _ in range(3)]
    m = torch.zeros_like(p)
    v = torch.zeros_like(p)
    pd, md, vd = p.to(cuda_dev), m.to(cuda_dev), v.to(cuda_dev)
    lr, b1, b2, eps, wd = 2e-4, 0.9, 0.999, 1e-8, 0.01
    for t, gr in enumerate(grads, start=1):
        total = float(gr.norm())
        coef = 1.0 / (total + 1e-6) if total > 1.0 else 1.0
        gc = gr * coef if total > 1.0 else gr
        m = b1 * m + (1 - b1) * gc
        v = b2 * v + (1 - b2) * gc * gc
        mh = m / (1 - b1 ** t)
        vh = v / (1 - b2 ** t)
        p = p - lr * (mh / (vh.sqrt() + eps) + wd * p)
        gd = gr.to(cuda_dev)
        clip = ops.grad_clip_coef(gd, 1.0)
        ops.adamw_step(pd, gd, md, vd, t, lr, b1, b2, eps, wd, clip=clip)
        assert abs(float(clip[0]) - total) / total < 1e-5
    assert torch.allclose(pd.cpu(), p, rtol=1e-5, atol=1e-7)


def test_fused_layer_kernels_vs_torch(cuda_dev):
    """RMSNorm / rotary / SwiGLU kernels (forward and gradient) against fp32
    torch restatements of the HF ops."""
    from fitllm_b200.layer import rotary_tables
    from fitllm_b200.layer_ops import rms_norm, rope, swiglu
    g = torch.Generator(device=cuda_dev).manual_seed(0)
    x = torch.randn(3, 40, 5120, generator=g, device=cuda_dev).bfloat16().requires_grad_(True)
    w = (1 + 0.1 * torch.randn(5120, generator=g, device=cuda_dev)).bfloat16()
    y = rms_norm(x, w, 1e-6)
    dy = torch.randn_like(y)
    y.backward(dy)
    xr = x.detach().float().requires_grad_(True)
    yr = w.float() * (xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-6))
    yr.backward(dy.float())
    assert onf4.rel_err(y.detach().float().cpu().numpy(), yr.detach().cpu().numpy()) < REL
    assert onf4.rel_err(x.grad.float().cpu().numpy(), xr.grad.cpu().numpy()) < REL

    heads, hd, S = 8, 128, 40
    t = torch.randn(3, S, heads * hd, generator=g, device=cuda_dev).bfloat16().requires_grad_(True)
    cos, sin = rotary_tables(S, hd, 1e6, cuda_dev)
    o = rope(t, cos, sin, heads)
    do = torch.randn_like(o)
    o.backward(do)
    tr = t.detach().float().view(3, S, heads, hd).requires_grad_(True)
    c = torch.cat([cos, cos], -1)[None, :, None, :]
    s = torch.cat([sin, sin], -1)[None, :, None, :]
    rot = torch.cat((-tr[..., hd // 2:], tr[..., : hd // 2]), -1)
    orf = tr * c + rot * s
    orf.backward(do.float().view(3, S, heads, hd))
    assert onf4.rel_err(o.detach().float().cpu().numpy(), orf.detach().reshape(3, S, -1).cpu().numpy()) < REL
    assert onf4.rel_err(t.grad.float().cpu().numpy(), tr.grad.reshape(3, S, -1).cpu().numpy()) < REL

    gate = torch.randn(4, 27648, generator=g, device=cuda_dev).bfloat16().requires_grad_(True)
    up = torch.randn(4, 27648, generator=g, device=cuda_dev).bfloat16().requires_grad_(True)
    a = swiglu(gate, up)
    da = torch.randn_like(a)
    a.backward(da)
    gr = gate.detach().float().requires_grad_(True)
    ur = up.detach().float().requires_grad_(True)
    ar = torch.nn.functional.silu(gr) * ur
    ar.backward(da.float())
    assert onf4.rel_err(a.detach().float().cpu().numpy(), ar.detach().cpu().numpy()) < REL
    assert onf4.rel_err(gate.grad.float().cpu().numpy(), gr.grad.cpu().numpy()) < REL
    assert onf4.rel_err(up.grad.float().cpu().numpy(), ur.grad.cpu().numpy()) < REL


@pytest.mark.parametrize("head_dim,heads,kv_heads,p", [(64, 4, 2, 16), (128, 8, 2, 100)])
def test_verify_pass_matches_full_forward(cuda_dev, head_dim, heads, kv_heads, p):
    """KV-cached verify (fitllm_b200/verify.py): filling the cache with the
    prefix, then running only the T new tokens of each sequence, gives the
    same last-T hidden states as the full causal forward over prefix + new
    tokens (the reference's re-prefill), within 1e-2.  head_dim 128 runs the
    verify step on fitq_verify_attention, head_dim 64 on torch SDPA."""
    from fitllm_b200.layer import DecoderLayer, LayerConfig, add_lora_, quantize_layer_
    from fitllm_b200.verify import KVCache, verify_pass
    cfg = LayerConfig(hidden=heads * head_dim, heads=heads, kv_heads=kv_heads, head_dim=head_dim,
                      intermediate=512)
    layers = []
    for i in range(2):
        layer = DecoderLayer(cfg, device=cuda_dev)
        quantize_layer_(layer, seed=40 + i)
        add_lora_(layer, 16, 32.0, ("q_proj", "v_proj"), seed=i, b_std=0.01)
        layer.eval()
        layers.append(layer)
    b, t = 2, 5
    g = torch.Generator(device=cuda_dev).manual_seed(9)
    h = torch.randn(b, p + t, cfg.hidden, generator=g, device=cuda_dev).bfloat16()
    with torch.no_grad():
        ref = h
        for layer in layers:
            ref = layer(ref)
        cache = KVCache(2, b, cfg.kv_heads, cfg.head_dim, p + t, cuda_dev)
        verify_pass(layers, h[:, :p].contiguous(), cache, prefix=0)
        out = verify_pass(layers, h[:, p:].contiguous(), cache, prefix=p)
    err = (out.float() - ref[:, p:].float()).norm() / ref[:, p:].float().norm()
    assert float(err) < 1e-2, float(err)


@pytest.mark.parametrize("group_size", [1, 2])
def test_engine_from_shard_files_matches_in_memory(cuda_dev, tmp_path, group_size):
    """A model read from FitLLM-format shard files (safetensors + .sha256,
    checksummed once at load) steps bit-identically to the same model built in
    memory; a corrupted file is refused before anything is stored."""
    from fitllm_b200 import shards
    from fitllm_b200.engine import (ShardStationaryEngine, build_model_from_shards,
                                    build_synthetic_model, synthetic_layer_shards)
    cfg = _cfg()
    shards.write_layer_shards(synthetic_layer_shards(cfg, 3, cuda_dev, seed=4), tmp_path,
                              group_size=group_size)
    g = torch.Generator().manual_seed(31)
    h = torch.randn(2, 64, SMALL["hidden"], generator=g).bfloat16().to(cuda_dev)
    go = torch.randn(2, 64, SMALL["hidden"], generator=g).bfloat16().to(cuda_dev)
    outs = []
    for build in ("memory", "files"):
        if build == "memory":
            sched, store = build_synthetic_model(cfg, 3, cuda_dev, seed=4)
        else:
            sched, store = build_model_from_shards(cfg, tmp_path, 3, cuda_dev, group_size=group_size,
                                                   seed=4)
        eng = ShardStationaryEngine(cfg, sched, store, cuda_dev, keep_activations=0)
        store.zero_grad()
        gin = eng.step(h, go)
        torch.cuda.synchronize()
        outs.append((gin.clone(), store.grad.clone()))
    assert torch.equal(outs[0][0], outs[1][0])
    assert torch.equal(outs[0][1], outs[1][1])
    first = tmp_path / shards.shard_file_name(0, 1 if group_size > 1 else None)
    raw = bytearray(first.read_bytes())
    raw[-1] ^= 0x5A
    first.write_bytes(bytes(raw))
    with pytest.raises(RuntimeError, match="Checksum mismatch"):
        build_model_from_shards(cfg, tmp_path, 3, cuda_dev, group_size=group_size)


def test_engine_step_with_lm_head_loss(cuda_dev):
    """The reference's full step (fitllm/trainer.py:495-535 with
    fitllm/backward.py:188-198): two layers streamed through the ring, the
    final norm + lm_head + CE loss of each micro-batch scaled by 1/grad_accum,
    backward.  Losses, input grad and LoRA grads against the fp32 CPU
    restatement with autograd, within 1e-2."""
    import torch.nn.functional as F
    from fitllm_b200.engine import ShardStationaryEngine, lora_entries
    from fitllm_b200.layer import DecoderLayer, add_lora_
    from fitllm_b200.lm_head import LMHeadLoss
    from fitllm_b200.optimizer import LoRAStore
    from fitllm_b200.scheduler import ShardScheduler
    cfg = _cfg()
    shards, refs = [], []
    for l in range(2):
        s, r = _oracle_shard(50 + l)
        shards.append(s)
        refs.append(r)
    sched = ShardScheduler(2, cuda_dev, ring_slots=2)
    for l in range(2):
        sched.add_layer(l, shards[l])
    proto = DecoderLayer(cfg, device=cuda_dev)
    add_lora_(proto, 16, 32.0, cfg.lora_targets, seed=0)
    store = LoRAStore(2, lora_entries(proto), cuda_dev)
    for l in range(2):
        store.init_layer_(l, {f"self_attn.{n}.lora_{ab}.default.weight": refs[l][f"{n}.lora_{ab}"]
                              for n in ("q_proj", "v_proj") for ab in ("A", "B")})
    vocab, nmb, seq = 2048, 2, 64
    g = torch.Generator().manual_seed(52)
    h = torch.randn(nmb, seq, SMALL["hidden"], generator=g).bfloat16()
    nw = (1 + 0.1 * torch.randn(SMALL["hidden"], generator=g)).bfloat16()
    w = (torch.randn(vocab, SMALL["hidden"], generator=g) * 0.05).bfloat16()
    labels = torch.randint(0, vocab, (nmb, seq), generator=g)
    labels[1, -5:] = -100
    head = LMHeadLoss(nw.to(cuda_dev), w.to(cuda_dev))
    eng = ShardStationaryEngine(cfg, sched, store, cuda_dev, keep_activations=1)
    store.zero_grad()
    losses, gin = eng.step_with_loss(h.to(cuda_dev), labels.to(cuda_dev), head, grad_accum=nmb)
    params = {l: {k: refs[l][k].clone().requires_grad_(True) for k in refs[l] if "lora_" in k}
              for l in range(2)}
    x = h.float().clone().requires_grad_(True)
    y = x
    for l in range(2):
        ww = dict(refs[l])
        ww.update(params[l])
        y = layer_ref.layer_forward(ww, y)
    z = nw.float() * (y * torch.rsqrt(y.pow(2).mean(-1, keepdim=True) + 1e-6))
    ref_losses = [F.cross_entropy(z[i] @ w.float().t(), labels[i], ignore_index=-100) for i in range(nmb)]
    (sum(ref_losses) / nmb).backward()
    for i in range(nmb):
        assert abs(float(losses[i]) - float(ref_losses[i].detach())) <= 1e-2 * float(ref_losses[i].detach())
    assert onf4.rel_err(gin.float().cpu().numpy(), x.grad.numpy()) < REL
    for l in range(2):
        gv = store.views(store.grad, l)
        for n in ("q_proj", "v_proj"):
            for ab in ("A", "B"):
                got = gv[f"self_attn.{n}.lora_{ab}.default.weight"].cpu().numpy()
                assert onf4.rel_err(got, params[l][f"{n}.lora_{ab}"].grad.numpy()) < REL


def test_rope_kv_append_matches_rope_and_copy(cuda_dev):
    """fitq_rope_append (one launch) gives the rotated q of the rope kernel and
    writes the rotated k and the v of the new tokens into the caches exactly
    where the unfused rope + cache copies put them, leaving the rest untouched."""
    from fitllm_b200.layer import rotary_tables
    from fitllm_b200.layer_ops import rope, rope_kv_append
    b, t, h, kvh, d, prefix, cap = 3, 5, 8, 2, 128, 37, 50
    g = torch.Generator(device=cuda_dev).manual_seed(61)
    q = torch.randn(b, t, h * d, generator=g, device=cuda_dev).bfloat16()
    k = torch.randn(b, t, kvh * d, generator=g, device=cuda_dev).bfloat16()
    v = torch.randn(b, t, kvh * d, generator=g, device=cuda_dev).bfloat16()
    cos, sin = rotary_tables(t, d, 1e6, cuda_dev, position_ids=torch.arange(prefix, prefix + t, device=cuda_dev))
    kc = torch.randn(b, kvh, cap, d, generator=g, device=cuda_dev).bfloat16()
    vc = torch.randn(b, kvh, cap, d, generator=g, device=cuda_dev).bfloat16()
    kc_ref, vc_ref = kc.clone(), vc.clone()
    with torch.no_grad():
        q_ref = rope(q, cos, sin, h).view(b, t, h, d)
        k_rot = rope(k, cos, sin, kvh).view(b, t, kvh, d)
    kc_ref[:, :, prefix:prefix + t] = k_rot.transpose(1, 2)
    vc_ref[:, :, prefix:prefix + t] = v.view(b, t, kvh, d).transpose(1, 2)
    q_out = rope_kv_append(q, k, v, cos, sin, kc, vc, prefix, h, kvh)
    torch.cuda.synchronize()
    assert torch.equal(q_out, q_ref)
    assert torch.equal(kc, kc_ref) and torch.equal(vc, vc_ref)


def test_host_batch_pipeline_matches_serial_steps(cuda_dev):
    """Engine steps fed through HostBatchPipeline (next batch's H2D and the
    previous result's D2H on their own streams, overlapping the step) return
    bit-identically what the same steps return with the copies in stream
    order, for batches that differ per step."""
    from fitllm_b200.engine import ShardStationaryEngine, build_synthetic_model
    from fitllm_b200.host_io import HostBatchPipeline
    cfg = _cfg()
    g = torch.Generator().manual_seed(41)
    shape = (2, 64, SMALL["hidden"])
    batches = [(torch.randn(*shape, generator=g).bfloat16().pin_memory(),
                torch.randn(*shape, generator=g).bfloat16().pin_memory()) for _ in range(4)]
    results = []
    for mode in ("serial", "pipeline"):
        sched, store = build_synthetic_model(cfg, 2, cuda_dev, seed=5)
        eng = ShardStationaryEngine(cfg, sched, store, cuda_dev, keep_activations=0)

        def step(bufs):
            store.zero_grad()
            gin = eng.step(bufs[0], bufs[1])
            return [gin, store.grad.clone()]

        outs = [(torch.empty(shape, dtype=torch.bfloat16).pin_memory(),
                 torch.empty(store.grad.shape, dtype=torch.float32).pin_memory()) for _ in batches]
        if mode == "serial":
            for (h, go), (o_gin, o_grad) in zip(batches, outs):
                gin, grad = step([h.to(cuda_dev), go.to(cuda_dev)])
                o_gin.copy_(gin)
                o_grad.copy_(grad)
        else:
            pipe = HostBatchPipeline(cuda_dev, batches[0])
            pipe.run(step, batches, outs)
            torch.cuda.synchronize()
            assert pipe.h2d_bytes == sum(t.numel() * t.element_size() for b in batches for t in b)
        results.append(outs)
    for (a_gin, a_grad), (b_gin, b_grad) in zip(*results):
        assert torch.equal(a_gin, b_gin)
        assert torch.equal(a_grad, b_grad)
    assert not torch.equal(results[1][0][0], results[1][1][0])  # the batches really differ


def test_reupload_into_rotated_slot_matches(cuda_dev):
    """One-layer engine steps with the shard re-uploaded every step: queued
    right after the previous step into the ring's other slot (invalidate +
    prefetch, the pipelined upload) they return bit-identically what steps
    with the upload in stream order return."""
    from fitllm_b200.engine import ShardStationaryEngine, build_synthetic_model
    cfg = _cfg()
    g = torch.Generator().manual_seed(43)
    shape = (2, 64, SMALL["hidden"])
    batches = [(torch.randn(*shape, generator=g).bfloat16().to(cuda_dev),
                torch.randn(*shape, generator=g).bfloat16().to(cuda_dev)) for _ in range(4)]
    results = []
    for mode in ("in_order", "rotated"):
        sched, store = build_synthetic_model(cfg, 1, cuda_dev, seed=6)
        eng = ShardStationaryEngine(cfg, sched, store, cuda_dev, keep_activations=0)
        outs = []
        for h, go in batches:
            if mode == "in_order":
                sched.invalidate()
            store.zero_grad()
            gin = eng.step(h, go)
            outs.append((gin.clone(), store.grad.clone()))
            if mode == "rotated":
                sched.invalidate()
                sched.prefetch(0)
        sched.wait_uploads()
        torch.cuda.synchronize()
        results.append(outs)
    for (a_gin, a_grad), (b_gin, b_grad) in zip(*results):
        assert torch.equal(a_gin, b_gin)
        assert torch.equal(a_grad, b_grad)
