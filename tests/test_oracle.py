"""CPU checks of the oracle itself (no GPU): the two restatements agree, the
NF4 table matches its published construction, the pinned vectors reproduce,
and the quantiser has the properties the format promises."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import nf4 as onf4

GOLD = Path(__file__).resolve().parent / "golden"


def test_nf4_levels_match_published_construction():
    # rebuilt from the N(0,1) quantile construction, equal to fp32 rounding
    assert np.allclose(onf4.normal_map_from_quantiles(), onf4.NF4_LEVELS, rtol=0, atol=2e-7)
    assert onf4.NF4_LEVELS[7] == 0.0 and onf4.NF4_LEVELS[0] == -1.0 and onf4.NF4_LEVELS[15] == 1.0
    assert np.all(np.diff(onf4.NF4_LEVELS) > 0)


def test_dynamic_map_shape_and_order():
    dm = onf4.dynamic_map_signed()
    assert dm.shape == (256,) and np.all(np.diff(dm) > 0)
    assert dm[-1] == 1.0 and 0.0 in dm
    assert np.isclose(dm[0], -0.99296875, atol=1e-6)


def test_product_tables_equal_oracle_tables():
    from fitllm_b200.nf4 import NF4_LEVELS, dynamic_quant_map
    assert np.array_equal(np.array(NF4_LEVELS, np.float32), onf4.NF4_LEVELS)
    assert np.array_equal(dynamic_quant_map().numpy(), onf4.dynamic_map_signed())


@pytest.mark.parametrize("shape", [(64, 64), (128, 320), (7, 4096)])
def test_c_and_numpy_restatements_agree(shape):
    g = torch.Generator().manual_seed(sum(shape))
    w = (torch.randn(*shape, generator=g) * 0.02).numpy()
    a, b = onf4.quantize(w), onf4.quantize_np(w)
    assert np.array_equal(a.packed, b.packed)
    assert np.array_equal(a.absmax_code, b.absmax_code)
    assert np.array_equal(a.nested_absmax, b.nested_absmax)
    assert a.offset == b.offset
    assert np.array_equal(onf4.dequant(a).reshape(-1), onf4.dequant_np(a).reshape(-1))


def test_pinned_vectors_reproduce():
    d = np.load(GOLD / "nf4_vectors.npz")
    st = onf4.quantize(d["w"])
    assert np.array_equal(st.packed, d["packed"])
    assert np.array_equal(st.absmax_code, d["absmax_code"])
    assert np.array_equal(st.nested_absmax, d["nested_absmax"])
    assert st.offset == d["offset"]
    assert np.array_equal(onf4.dequant(st, "bf16"), d["dequant_bf16"])
    assert np.array_equal(onf4.dequant(st, "f16"), d["dequant_f16"])


def test_quantiser_properties():
    d = np.load(GOLD / "nf4_vectors.npz")
    w = d["w"]
    st = onf4.quantize(w)
    deq = onf4.bf16_bits_to_f32(onf4.dequant(st, "bf16"))
    # all-zero block decodes to exact zeros of level 7
    assert np.all(deq[0, :64] == 0.0)
    nib = np.empty(w.size, np.uint8)
    nib[0::2], nib[1::2] = st.packed >> 4, st.packed & 15
    assert np.all(nib.reshape(w.shape)[0, :64] == 7)
    # exact-level block: every element picks its own level
    assert np.array_equal(nib.reshape(w.shape)[1, :64], np.arange(64) % 16)
    # |w - q.am_dec| <= gap.am_true + |am_true - am_dec|  (gap: half the widest level gap)
    am_dec = onf4.absmax_decode(st)
    am_true = np.abs(w).reshape(-1, 64).max(axis=1)
    gap = np.max(np.diff(onf4.NF4_LEVELS)) / 2
    err = np.abs(deq - w).reshape(-1, 64).max(axis=1)
    bound = gap * am_true + np.abs(am_true - am_dec)
    assert np.all(err <= bound * (1 + 1e-2) + 1e-7)


def test_f16_and_bf16_conversions_are_rne():
    L = onf4.lib()
    x = np.array([1.0, 1 + 2 ** -8, 1 + 3 * 2 ** -9, 65519.0, 65520.0, 6e-8, 3e-8, -0.0,
                  np.inf, -np.inf], np.float32)
    got16 = np.array([L.oracle_f32_to_f16(float(v)) for v in x], np.uint16)
    assert np.array_equal(got16, x.astype(np.float16).view(np.uint16))
    gotb = np.array([L.oracle_f32_to_bf16(float(v)) for v in x], np.uint16)
    ref = torch.from_numpy(x).bfloat16().view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(gotb, ref)


def test_qlora_reference_math_consistency():
    """Finite-difference check of the fp64 QLoRA backward restatement."""
    g = np.random.default_rng(0)
    m, n, k, r = 5, 7, 6, 2
    x, w = g.standard_normal((m, k)), g.standard_normal((n, k))
    A, B, dy = g.standard_normal((r, k)), g.standard_normal((n, r)), g.standard_normal((m, n))
    s = 1.5
    dX, dA, dB = onf4.qlora_backward(x, w, A, B, s, dy)
    f = lambda xx, AA, BB: float(np.sum(onf4.qlora_forward(xx, w, AA, BB, s) * dy))
    eps = 1e-6
    for arr, grad, name in ((x, dX, "x"), (A, dA, "A"), (B, dB, "B")):
        num = np.zeros_like(arr)
        for idx in np.ndindex(arr.shape):
            p = arr.copy(); p[idx] += eps
            q = arr.copy(); q[idx] -= eps
            args = {"x": (x, A, B), "A": (x, A, B), "B": (x, A, B)}[name]
            fp = f(*(p if i == ["x", "A", "B"].index(name) else v for i, v in enumerate(args)))
            fm = f(*(q if i == ["x", "A", "B"].index(name) else v for i, v in enumerate(args)))
            num[idx] = (fp - fm) / (2 * eps)
        assert np.allclose(num, grad, rtol=1e-5, atol=1e-6), name


def test_torch_dequant_matches_oracle_bits():
    """The multi-threaded torch restatement of the dequant (used by the timed
    CPU baselines) gives the C oracle's values bit for bit."""
    from oracle import nf4 as onf4
    import torch
    w = (torch.randn(192, 640, generator=torch.Generator().manual_seed(4)) * 0.02).numpy()
    w[3, :64] = 0.0
    st = onf4.quantize(w)
    got = onf4.dequant_torch(st).numpy().view(np.uint32)
    ref = onf4.bf16_bits_to_f32(onf4.dequant(st, "bf16")).view(np.uint32)
    assert np.array_equal(got, ref)
