"""Causal GQA attention of the training layer (fitq_attention_fwd / _bwd).

The kernels replace the attention inside the Qwen2 decoder layer that FitLLM
runs in its shard-stationary forward and backward recompute
(fitllm/forward.py:657-701, fitllm/backward.py:222-231).  The reference for
every check is the same attention restated in fp32 torch from the same bf16
inputs: softmax(q k^T / sqrt(128) + causal mask) v with query head h reading
KV head h // (H / KVH), and its autograd gradients.  Tolerance: 1e-2 relative
(norm-wise), the bar the projections are held to.
"""
import json
import math

import pytest
import torch

from oracle import layer_ref
from oracle import nf4 as onf4

pytestmark = pytest.mark.gpu
REL = 1e-2
FITQ_ERR_SHAPE, FITQ_ERR_ALIGN, FITQ_ERR_UNSUPPORTED = 2, 3, 4


def _rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm())


def _ref_attention(q, k, v):
    """fp32 restatement over [B, S, H, D] / [B, S, KVH, D]: (o, lse in nats)."""
    b, s, h, d = q.shape
    grp = h // k.shape[2]
    qf = q.float().transpose(1, 2)
    kf = k.float().transpose(1, 2).repeat_interleave(grp, dim=1)
    vf = v.float().transpose(1, 2).repeat_interleave(grp, dim=1)
    sc = qf @ kf.transpose(-1, -2) / math.sqrt(d)
    mask = torch.ones(s, s, dtype=torch.bool, device=q.device).triu(1)
    sc = sc.masked_fill(mask, float("-inf"))
    lse = torch.logsumexp(sc, dim=-1)
    o = torch.softmax(sc, dim=-1) @ vf
    return o.transpose(1, 2), lse


def _inputs(b, s, h, kvh, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn(b, s, h, 128, generator=g, device=dev).bfloat16()
    k = torch.randn(b, s, kvh, 128, generator=g, device=dev).bfloat16()
    v = torch.randn(b, s, kvh, 128, generator=g, device=dev).bfloat16()
    do = torch.randn(b, s, h, 128, generator=g, device=dev).bfloat16()
    return q, k, v, do


SHAPES = [(1, 64, 1, 1), (2, 256, 10, 2), (1, 512, 40, 8), (2, 192, 4, 4), (1, 2048, 40, 8)]


@pytest.mark.parametrize("b,s,h,kvh", SHAPES)
def test_attention_forward_matches_fp32(cuda_dev, b, s, h, kvh):
    from fitllm_b200.layer_ops import attention_forward
    q, k, v, _ = _inputs(b, s, h, kvh, 1 + s + h, cuda_dev)
    o, lse = attention_forward(q, k, v)
    torch.cuda.synchronize()
    ro, rlse = _ref_attention(q, k, v)
    assert _rel(o.float(), ro) < REL
    # lse is kept in base-2 units of the scaled scores
    assert torch.allclose(lse, rlse.float() / math.log(2.0), rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("b,s,h,kvh", SHAPES)
def test_attention_backward_matches_fp32(cuda_dev, b, s, h, kvh):
    from fitllm_b200.layer_ops import attention_backward, attention_forward
    q, k, v, do = _inputs(b, s, h, kvh, 7 + s + h, cuda_dev)
    o, lse = attention_forward(q, k, v)
    dq, dk, dv = attention_backward(q, k, v, o, lse, do)
    torch.cuda.synchronize()
    qf, kf, vf = (t.float().requires_grad_(True) for t in (q, k, v))
    ro, _ = _ref_attention(qf, kf, vf)
    ro.backward(do.float())
    assert _rel(dq.float(), qf.grad) < REL
    assert _rel(dk.float(), kf.grad) < REL
    assert _rel(dv.float(), vf.grad) < REL


def test_attention_is_deterministic(cuda_dev):
    from fitllm_b200.layer_ops import attention_backward, attention_forward
    q, k, v, do = _inputs(2, 256, 10, 2, 3, cuda_dev)
    runs = []
    for _ in range(2):
        o, lse = attention_forward(q, k, v)
        runs.append((o, lse) + attention_backward(q, k, v, o, lse, do))
    torch.cuda.synchronize()
    for a, c in zip(*runs):
        assert torch.equal(a, c)


def test_attention_autograd_function(cuda_dev):
    from fitllm_b200.layer_ops import attention
    q, k, v, do = _inputs(1, 128, 4, 2, 5, cuda_dev)
    qa, ka, va = (t.clone().requires_grad_(True) for t in (q, k, v))
    o = attention(qa, ka, va)
    o.backward(do)
    qf, kf, vf = (t.float().requires_grad_(True) for t in (q, k, v))
    ro, _ = _ref_attention(qf, kf, vf)
    ro.backward(do.float())
    assert _rel(o.detach().float(), ro.detach()) < REL
    for got, ref in ((qa.grad, qf.grad), (ka.grad, kf.grad), (va.grad, vf.grad)):
        assert got.dtype == torch.bfloat16
        assert _rel(got.float(), ref) < REL


def test_attention_refuses_bad_calls_on_host(cuda_dev):
    """Shapes and pointers the kernels do not take come back as status codes
    before anything is launched."""
    from fitllm_b200 import _lib
    L = _lib.load()
    st = torch.cuda.current_stream().cuda_stream
    buf = torch.zeros(1 << 20, dtype=torch.bfloat16, device=cuda_dev)
    lse = torch.zeros(1 << 16, dtype=torch.float32, device=cuda_dev)
    p, pl = buf.data_ptr(), lse.data_ptr()
    torch.cuda.synchronize()
    before = L.fitq_launch_count()
    assert L.fitq_attention_fwd(p, p, p, p, pl, 1, 100, 4, 2, 128, st) == FITQ_ERR_SHAPE  # S % 64
    assert L.fitq_attention_fwd(p, p, p, p, pl, 1, 128, 5, 2, 128, st) == FITQ_ERR_SHAPE  # H % KVH
    assert L.fitq_attention_fwd(p, p, p, p, pl, 1, 128, 4, 2, 64, st) == FITQ_ERR_UNSUPPORTED
    assert L.fitq_attention_fwd(p + 2, p, p, p, pl, 1, 128, 4, 2, 128, st) == FITQ_ERR_ALIGN
    ws = L.fitq_attention_bwd_workspace(1, 128, 4)
    assert ws == 128 * 4 * 4
    assert L.fitq_attention_bwd(p, p, p, p, p, pl, p, p, p, 1, 128, 4, 2, 128, pl, ws - 4, st) == 5
    assert L.fitq_launch_count() == before
    assert b"attention" in L.fitq_last_error()


# A decoder layer with head_dim 128 (the size the kernels take), the kernel
# switched on, against the oracle's fp32 CPU restatement of the whole layer.
DIMS = dict(hidden=512, heads=4, kv_heads=2, head_dim=128, inter=512)


def _shard(seed):
    g = torch.Generator().manual_seed(seed)
    shard, ref = {}, {}
    names = {"q_proj": "self_attn", "k_proj": "self_attn", "v_proj": "self_attn",
             "o_proj": "self_attn", "gate_proj": "mlp", "up_proj": "mlp", "down_proj": "mlp"}
    for name, kind, bias in layer_ref.PROJ:
        n, k = layer_ref.proj_shape(kind, DIMS["hidden"], DIMS["heads"], DIMS["kv_heads"],
                                    DIMS["head_dim"], DIMS["inter"])
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
    shard["input_layernorm.weight"] = torch.ones(DIMS["hidden"], dtype=torch.bfloat16)
    shard["post_attention_layernorm.weight"] = torch.ones(DIMS["hidden"], dtype=torch.bfloat16)
    for name in ("q_proj", "v_proj"):
        n, k = ref[name].shape
        ref[name + ".lora_A"] = (torch.rand(16, k, generator=g) * 2 - 1) / math.sqrt(k)
        ref[name + ".lora_B"] = torch.randn(n, 16, generator=g) * 0.02
    ref["scale"] = torch.tensor(2.0)
    ref["cfg"] = torch.tensor([DIMS["hidden"], DIMS["heads"], DIMS["kv_heads"], DIMS["head_dim"],
                               DIMS["inter"]])
    return shard, ref


def test_decoder_layer_with_attention_kernel_vs_restatement(cuda_dev, monkeypatch):
    from fitllm_b200.layer import DecoderLayer, LayerConfig, add_lora_
    monkeypatch.setenv("FITQ_ATTN", "1")
    cfg = LayerConfig(hidden=DIMS["hidden"], heads=DIMS["heads"], kv_heads=DIMS["kv_heads"],
                      head_dim=DIMS["head_dim"], intermediate=DIMS["inter"], lora_rank=16,
                      lora_alpha=32.0, lora_targets=("q_proj", "v_proj"))
    shard, ref = _shard(21)
    layer = DecoderLayer(cfg, device=cuda_dev)
    assert layer.self_attn.own_kernel
    layer.load_state_dict(shard, strict=False)
    add_lora_(layer, 16, 32.0, ("q_proj", "v_proj"), seed=0)
    with torch.no_grad():
        for name in ("q_proj", "v_proj"):
            mod = layer.self_attn.get_submodule(name)
            mod.lora_A["default"].weight.copy_(ref[name + ".lora_A"])
            mod.lora_B["default"].weight.copy_(ref[name + ".lora_B"])
    g = torch.Generator().manual_seed(22)
    h = torch.randn(2, 128, DIMS["hidden"], generator=g).bfloat16()
    go = torch.randn(2, 128, DIMS["hidden"], generator=g).bfloat16()
    hd = h.to(cuda_dev).requires_grad_(True)
    before = _launches()
    y = layer(hd)
    y.backward(go.to(cuda_dev))
    torch.cuda.synchronize()
    assert _launches() > before
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


def _launches():
    from fitllm_b200 import _lib
    return _lib.load().fitq_launch_count()
