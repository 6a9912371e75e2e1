"""fitq_lora_merge on the GPU: bit-exact against the oracle for bf16, fp16
and fp32 weights at the q_proj / v_proj shapes, NF4 weights merged and
re-quantised bit-exactly against the C oracle, and the shard-file merge of
fitllm/inference.py:79-144 end to end."""
import numpy as np
import pytest
import torch

from oracle import merge as omerge
from oracle import nf4 as onf4

pytestmark = pytest.mark.gpu


def _state_to_device(st, dev):
    from fitllm_b200.nf4 import QuantState
    packed = torch.from_numpy(st.packed.copy()).to(dev).view(-1, 1)
    qs = QuantState(absmax=torch.from_numpy(st.absmax_code.copy()).to(dev), shape=st.shape,
                    quant_map=torch.from_numpy(st.quant_map.copy()).to(dev),
                    nested_absmax=torch.from_numpy(st.nested_absmax.copy()).to(dev),
                    nested_quant_map=torch.from_numpy(st.nested_quant_map.copy()).to(dev),
                    offset=float(st.offset))
    return packed, qs


def _case(n, k, r, seed):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=g) * 0.02
    a = (torch.rand(r, k, generator=g) * 2 - 1) / np.sqrt(k)
    b = torch.randn(n, r, generator=g) * 0.01
    return w, a, b


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("n,k,r", [(5120, 5120, 16), (1024, 5120, 16), (100, 1000, 37), (17, 34, 64),
                                   (48, 2048, 1), (16, 512, 256)])
def test_lora_merge_bit_exact(cuda_dev, dtype, n, k, r):
    from fitllm_b200.merge import lora_merge_
    w, a, b = _case(n, k, r, n * 7 + r)
    w = w.to(dtype)
    s = 32.0 / 16
    out = lora_merge_(w.to(cuda_dev).contiguous(), a.to(cuda_dev), b.to(cuda_dev), s).cpu()
    if dtype == torch.bfloat16:
        ref = omerge.merge_bf16_bits(w.view(torch.int16).numpy().view(np.uint16), a.numpy(), b.numpy(), s)
        assert np.array_equal(out.view(torch.int16).numpy().view(np.uint16), ref)
    elif dtype == torch.float16:
        ref = omerge.merge_f16(w.numpy(), a.numpy(), b.numpy(), s)
        assert np.array_equal(out.numpy().view(np.uint16), ref.view(np.uint16))
    else:
        ref = omerge.merge_f32(w.numpy(), a.numpy(), b.numpy(), s)
        assert np.array_equal(out.numpy().view(np.uint32), ref.view(np.uint32))


def test_lora_merge_rejects_bad_arguments(cuda_dev):
    from fitllm_b200 import _lib
    L = _lib.load()
    w = torch.zeros(8, 6, dtype=torch.bfloat16, device=cuda_dev)
    a = torch.zeros(2, 6, device=cuda_dev)
    b = torch.zeros(8, 2, device=cuda_dev)
    st = torch.cuda.current_stream().cuda_stream
    assert L.fitq_lora_merge(w.data_ptr(), 0, 8, 5, a.data_ptr(), b.data_ptr(), 2, 1.0, st) == 2
    assert L.fitq_lora_merge(w.data_ptr(), 0, 8, 6, a.data_ptr(), b.data_ptr(), 0, 1.0, st) == 2
    assert L.fitq_lora_merge(w.data_ptr(), 7, 8, 6, a.data_ptr(), b.data_ptr(), 2, 1.0, st) == 1
    assert L.fitq_lora_merge(w.data_ptr() + 2, 0, 8, 6, a.data_ptr(), b.data_ptr(), 2, 1.0, st) == 3
    assert L.fitq_lora_merge(None, 0, 8, 6, a.data_ptr(), b.data_ptr(), 2, 1.0, st) == 1


@pytest.mark.parametrize("n,k,r", [(1024, 5120, 16), (192, 640, 8)])
def test_nf4_merge_bit_exact(cuda_dev, n, k, r):
    """dequant (bit-exact) -> merge -> re-quantise, against the C oracle's
    dequant, the merge restatement and the C oracle's quantiser."""
    from fitllm_b200.merge import merge_nf4
    w, a, b = _case(n, k, r, n + r)
    st = onf4.quantize(w.numpy())
    packed, qs = _state_to_device(st, cuda_dev)
    s = 2.0
    p2, qs2 = merge_nf4(packed, qs, a.to(cuda_dev), b.to(cuda_dev), s)
    merged_bits = omerge.merge_bf16_bits(onf4.dequant(st, "bf16"), a.numpy(), b.numpy(), s)
    ref = onf4.quantize(onf4.bf16_bits_to_f32(merged_bits), st.quant_map, st.nested_quant_map)
    assert np.array_equal(p2.view(-1).cpu().numpy(), ref.packed)
    assert np.array_equal(qs2.absmax.cpu().numpy(), ref.absmax_code)
    assert np.array_equal(qs2.nested_absmax.cpu().numpy(), ref.nested_absmax)
    assert np.float32(qs2.offset) == ref.offset


def test_merge_lora_into_shards_end_to_end(cuda_dev, tmp_path):
    """One layer shard with a dense bf16 q_proj, an NF4 v_proj (flat bnb keys)
    and PEFT adapters on both, plus an untouched o_proj: merged in place,
    adapters dropped, checksum rewritten."""
    from fitllm_b200.merge import merge_lora_into_shards
    from fitllm_b200.nf4 import QuantState, quantize_nf4, dequantize_nf4
    from fitllm_b200.shards import load_shard_with_checksum, save_shard_with_checksum, verify_shard
    hidden, r = 256, 16
    wq, aq, bq = _case(hidden, hidden, r, 1)
    wv, av, bv = _case(64, hidden, r, 2)
    wo, _, _ = _case(hidden, hidden, r, 3)
    packed, qs = quantize_nf4(wv.to(cuda_dev))
    sd = {"self_attn.q_proj.weight": wq.bfloat16(),
          "self_attn.q_proj.lora_A.default.weight": aq, "self_attn.q_proj.lora_B.default.weight": bq,
          "self_attn.v_proj.weight": packed.cpu(),
          "self_attn.v_proj.lora_A.default.weight": av, "self_attn.v_proj.lora_B.default.weight": bv,
          "self_attn.o_proj.weight": wo.bfloat16()}
    for kk, v in qs.as_dict(packed=True).items():
        sd[f"self_attn.v_proj.weight.{kk}"] = v.cpu()
    path = tmp_path / "layer_000.safetensors"
    save_shard_with_checksum(sd, path)
    done = merge_lora_into_shards([path], rank=r, alpha=32.0, device=cuda_dev)
    assert sorted(done[str(path)]) == ["self_attn.q_proj.weight", "self_attn.v_proj.weight"]
    verify_shard(path)
    out = load_shard_with_checksum(path)
    assert not any("lora_" in kk for kk in out)
    s = 32.0 / r
    q_ref = omerge.merge_bf16_bits(wq.bfloat16().view(torch.int16).numpy().view(np.uint16), aq.numpy(),
                                   bq.numpy(), s)
    assert np.array_equal(out["self_attn.q_proj.weight"].view(torch.int16).numpy().view(np.uint16), q_ref)
    assert torch.equal(out["self_attn.o_proj.weight"], wo.bfloat16())
    flat = {kk[len("self_attn.v_proj.weight."):]: v for kk, v in out.items()
            if kk.startswith("self_attn.v_proj.weight.")}
    qs2 = QuantState.from_dict(flat, device=cuda_dev)
    v_deq = dequantize_nf4(out["self_attn.v_proj.weight"].to(cuda_dev), qs2).float().cpu()
    v_dense = omerge.reference_formula(dequantize_nf4(packed, qs).cpu(), av, bv, s).float()
    # re-quantised: within NF4's own rounding of the merged weight
    assert float((v_deq - v_dense).norm() / v_dense.norm()) < 0.12
