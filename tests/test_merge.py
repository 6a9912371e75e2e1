"""LoRA merge (fitllm/inference.py:79-144): the oracle against the
reference's own torch expression, and the shard-key logic, on CPU."""
import numpy as np
import pytest
import torch

from oracle import merge as omerge
from oracle import nf4 as onf4


def _case(n, k, r, seed, scale_w=0.02):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=g) * scale_w
    a = (torch.rand(r, k, generator=g) * 2 - 1) / np.sqrt(k)
    b = torch.randn(n, r, generator=g) * 0.01
    return w, a, b


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("n,k,r", [(64, 256, 16), (33, 130, 8), (128, 512, 64)])
def test_oracle_matches_reference_formula(dtype, n, k, r):
    """The fixed-order restatement equals (W.float() + s * (B @ A)).to(dtype)
    except where torch's sum order moves the fp32 value across a rounding
    boundary of the output dtype: then by one unit in the last place."""
    w, a, b = _case(n, k, r, n + k + r)
    w = w.to(dtype)
    s = 32.0 / r
    ref = omerge.reference_formula(w, a, b, s)
    if dtype == torch.bfloat16:
        bits = w.view(torch.int16).numpy().view(np.uint16)
        got = omerge.merge_bf16_bits(bits, a.numpy(), b.numpy(), s)
        ref_bits = ref.view(torch.int16).numpy().view(np.uint16)
        ulp = np.abs(got.astype(np.int32) - ref_bits.astype(np.int32))
    elif dtype == torch.float16:
        got = omerge.merge_f16(w.numpy(), a.numpy(), b.numpy(), s)
        ulp = np.abs(got.view(np.int16).astype(np.int32) - ref.numpy().view(np.int16).astype(np.int32))
    else:
        got = omerge.merge_f32(w.numpy(), a.numpy(), b.numpy(), s)
        # fp32: the two rank-sum orders differ by at most r roundings of the
        # terms' magnitudes, plus the final rounding
        bound = (r + 2) * 2.0 ** -24 * (s * (np.abs(b.numpy()) @ np.abs(a.numpy())) + np.abs(w.numpy()))
        assert np.all(np.abs(got.astype(np.float64) - ref.numpy().astype(np.float64)) <= bound)
        return
    assert ulp.max() <= 1
    assert (ulp == 0).mean() > 0.99


def test_oracle_rank_sum_order():
    """Rank order with rounded products and sums, checked on values where
    a fused multiply-add or a different order would differ."""
    a = np.array([[1.0], [2.0 ** -24], [2.0 ** -24]], np.float32)
    b = np.array([[1.0, 1.0, 1.0]], np.float32)
    t = omerge.rank_sum(a, b)
    assert t[0, 0] == np.float32(1.0)  # 1 + 2^-24 rounds to 1, twice


def test_lora_pair_and_layout_logic():
    from fitllm_b200.merge import _lora_pair, _peft_layout
    t = {"self_attn.q_proj.weight": torch.zeros(8, 4),
         "self_attn.q_proj.lora_A.default.weight": torch.zeros(2, 4),
         "self_attn.q_proj.lora_B.default.weight": torch.zeros(8, 2),
         "self_attn.v_proj.weight": torch.zeros(8, 4),
         "mlp.up_proj.weight": torch.zeros(8, 4)}
    assert _lora_pair(t, "self_attn.q_proj") == ("self_attn.q_proj.lora_A.default.weight",
                                                 "self_attn.q_proj.lora_B.default.weight")
    assert _lora_pair(t, "self_attn.v_proj") == (None, None)
    assert _lora_pair(t, "mlp.up_proj") == (None, None)
    a, b = _peft_layout(torch.zeros(2, 4), torch.zeros(8, 2), 8, 4)
    assert a.shape == (2, 4) and b.shape == (8, 2)
    a, b = _peft_layout(torch.zeros(4, 2), torch.zeros(2, 8), 8, 4)  # own LoRALinear layout
    assert a.shape == (2, 4) and b.shape == (8, 2)
    with pytest.raises(ValueError):
        _peft_layout(torch.zeros(3, 3), torch.zeros(3, 3), 8, 4)
