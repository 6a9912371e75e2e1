"""Parity of the sm_100a kernels (through the C ABI) with the CPU oracle.

Bit-exact: NF4 dequant (bf16 and fp16, plain and transposed), NF4 quantise.
Within the 1e-2 relative contract (||out - ref|| / ||ref||, bf16 in, fp32
accumulate): the tcgen05 GEMM, the QLoRA forward (GEMM and GEMV paths) and the
backward (dX, dA, dB).
"""
import math

import numpy as np
import pytest
import torch

from oracle import nf4 as onf4

pytestmark = pytest.mark.gpu

REL_TOL = 1e-2  # north-star output/gradient tolerance (relative Frobenius norm)


def _state_to_device(st, dev):
    from fitllm_b200.nf4 import QuantState
    packed = torch.from_numpy(st.packed.copy()).to(dev).view(-1, 1)
    qs = QuantState(
        absmax=torch.from_numpy(st.absmax_code.copy()).to(dev),
        shape=st.shape,
        quant_map=torch.from_numpy(st.quant_map.copy()).to(dev),
        nested_absmax=torch.from_numpy(st.nested_absmax.copy()).to(dev),
        nested_quant_map=torch.from_numpy(st.nested_quant_map.copy()).to(dev),
        offset=float(st.offset))
    return packed, qs


def _weights(n, k, seed, std=0.02):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n, k, generator=g) * std).numpy().astype(np.float32)


def _bf16(t):
    return t.to(torch.bfloat16)


@pytest.mark.parametrize("n,k", [(64, 64), (128, 320), (1024, 512), (192, 4096)])
def test_dequant_bit_exact(cuda_dev, n, k):
    from fitllm_b200.nf4 import dequantize_nf4
    st = onf4.quantize(_weights(n, k, 10 + n))
    packed, qs = _state_to_device(st, cuda_dev)
    ref = onf4.dequant(st, "bf16")
    out = dequantize_nf4(packed, qs, torch.bfloat16)
    got = out.view(torch.int16).cpu().numpy().view(np.uint16)
    assert np.array_equal(got, ref)
    ref16 = onf4.dequant(st, "f16")
    out16 = dequantize_nf4(packed, qs, torch.float16)
    assert np.array_equal(out16.view(torch.int16).cpu().numpy().view(np.uint16), ref16)
    outt = dequantize_nf4(packed, qs, torch.bfloat16, transpose=True)
    assert np.array_equal(outt.view(torch.int16).cpu().numpy().view(np.uint16), ref.T)


def test_dequant_plain_absmax(cuda_dev):
    """State without double quantisation (fp32 absmax)."""
    from fitllm_b200.nf4 import QuantState, dequantize_nf4
    n, k = 96, 256
    w = _weights(n, k, 3)
    st = onf4.quantize(w)
    absmax = onf4.absmax_decode(st)
    packed = torch.from_numpy(st.packed.copy()).to(cuda_dev)
    qs = QuantState(absmax=torch.from_numpy(absmax).to(cuda_dev), shape=(n, k),
                    quant_map=torch.from_numpy(st.quant_map.copy()).to(cuda_dev))
    out = dequantize_nf4(packed, qs).view(torch.int16).cpu().numpy().view(np.uint16)
    assert np.array_equal(out, onf4.dequant(st, "bf16"))


@pytest.mark.parametrize("n,k", [(64, 64), (256, 1024), (333 * 64 // 64, 64 * 70)])
def test_quantize_bit_exact(cuda_dev, n, k):
    from fitllm_b200.nf4 import quantize_nf4
    w = _weights(n, k, 100 + k)
    w[0, :64] = 0.0  # an all-zero block
    st = onf4.quantize(w)
    packed, qs = quantize_nf4(torch.from_numpy(w).to(cuda_dev))
    assert np.array_equal(packed.view(-1).cpu().numpy(), st.packed)
    assert np.array_equal(qs.absmax.cpu().numpy(), st.absmax_code)
    assert np.array_equal(qs.nested_absmax.cpu().numpy(), st.nested_absmax)
    assert np.float32(qs.offset) == st.offset


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (1, 16, 64), (300, 272, 192), (1024, 1024, 4096),
                                   (512, 1024, 512), (1000, 768, 1024)])
@pytest.mark.parametrize("variant", ["1cta", "2cta"])
def test_gemm_bf16_tn(cuda_dev, m, n, k, variant, monkeypatch):
    monkeypatch.setenv("FITQ_GEMM_VARIANT", variant)
    from fitllm_b200.ops import gemm_bf16_tn
    g = torch.Generator(device="cpu").manual_seed(m * 7 + n)
    a = _bf16(torch.randn(m, k, generator=g)).to(cuda_dev)
    b = _bf16(torch.randn(n, k, generator=g)).to(cuda_dev)
    c = gemm_bf16_tn(a, b)
    ref = a.float() @ b.float().T
    assert onf4.rel_err(c.float().cpu().numpy(), ref.cpu().numpy()) < 4e-3
    add = _bf16(torch.randn(m, n, generator=g)).to(cuda_dev)
    c2 = gemm_bf16_tn(a, b, add)
    assert onf4.rel_err(c2.float().cpu().numpy(), (ref + add.float()).cpu().numpy()) < 4e-3


@pytest.mark.parametrize("bn", [256, 192, 160, 144, 128])
@pytest.mark.parametrize("m,n,k", [(512, 5120, 512), (300, 272, 192), (1000, 1008, 320), (129, 144, 64)])
def test_gemm_one_cta_tile_widths(cuda_dev, m, n, k, bn, monkeypatch):
    """The one-CTA tcgen05 GEMM at every built tile width (ragged N tiles,
    ragged rows, bias + residual epilogue, the LoRA K block) against fp32."""
    monkeypatch.setenv("FITQ_GEMM_VARIANT", "1cta")
    monkeypatch.setenv("FITQ_GEMM_BN", str(bn))
    from fitllm_b200.ops import gemm_bf16_tn
    g = torch.Generator(device="cpu").manual_seed(m + n + bn)
    a = _bf16(torch.randn(m, k, generator=g)).to(cuda_dev)
    b = _bf16(torch.randn(n, k, generator=g)).to(cuda_dev)
    add = _bf16(torch.randn(m, n, generator=g)).to(cuda_dev)
    ref = a.float() @ b.float().T
    c = gemm_bf16_tn(a, b, add)
    assert onf4.rel_err(c.float().cpu().numpy(), (ref + add.float()).cpu().numpy()) < 4e-3


@pytest.mark.parametrize("bn", [256, 192, 160, 144, 128])
@pytest.mark.parametrize("m,n,k", [(512, 5120, 512), (300, 272, 192), (1000, 1008, 320), (600, 144, 64)])
def test_gemm_pair_tile_widths(cuda_dev, m, n, k, bn, monkeypatch):
    """The CTA-pair tcgen05 GEMM at every built tile width (each CTA loads
    bn / 2 rows of B; ragged N tiles and rows; residual epilogue)."""
    monkeypatch.setenv("FITQ_GEMM_VARIANT", "2cta")
    monkeypatch.setenv("FITQ_GEMM_BN2", str(bn))
    from fitllm_b200.ops import gemm_bf16_tn
    g = torch.Generator(device="cpu").manual_seed(m + n + bn + 1)
    a = _bf16(torch.randn(m, k, generator=g)).to(cuda_dev)
    b = _bf16(torch.randn(n, k, generator=g)).to(cuda_dev)
    add = _bf16(torch.randn(m, n, generator=g)).to(cuda_dev)
    ref = a.float() @ b.float().T
    c = gemm_bf16_tn(a, b, add)
    assert onf4.rel_err(c.float().cpu().numpy(), (ref + add.float()).cpu().numpy()) < 4e-3


@pytest.mark.parametrize("variant,env,bn", [("1cta", "FITQ_GEMM_BN", 144), ("2cta", "FITQ_GEMM_BN2", 144),
                                            ("2cta", "FITQ_GEMM_BN2", 192)])
def test_qlora_tile_widths_identical(cuda_dev, variant, env, bn, monkeypatch):
    """QLoRA fwd / bwd at the q_proj shape: the tile width changes the
    schedule, not the arithmetic (every output element's K sum is the same
    sequence of MMAs), so y and dX are bit-identical across widths."""
    from fitllm_b200 import ops
    monkeypatch.setenv("FITQ_NF4_FUSED", "0")
    monkeypatch.setenv("FITQ_GEMM_VARIANT", variant)
    st, wref, w_deq, A, B, x, dy = _qlora_case(512, 5120, 5120, 16, 77, cuda_dev)
    Ad, Bd, xd, dyd = A.to(cuda_dev), B.to(cuda_dev), x.to(cuda_dev), dy.to(cuda_dev)
    out = {}
    for w in (256, bn):
        monkeypatch.setenv(env, str(w))
        y, t = ops.qlora_forward(xd, wref, Ad, Bd, 2.0, want_t=True)
        dx, ga, gb = ops.qlora_backward(xd, dyd, wref, Ad, Bd, 2.0, t_saved=t)
        out[w] = (y, dx, ga, gb)
    torch.cuda.synchronize()
    for i in range(4):
        assert torch.equal(out[256][i], out[bn][i])


def _qlora_case(m, n, k, r, seed, dev):
    from fitllm_b200.nf4 import Nf4WeightCRef
    st = onf4.quantize(_weights(n, k, seed))
    packed, qs = _state_to_device(st, dev)
    w_deq = onf4.bf16_bits_to_f32(onf4.dequant(st, "bf16"))
    g = torch.Generator().manual_seed(seed + 1)
    bound = 1.0 / np.sqrt(k)  # kaiming_uniform(a=sqrt(5)) bound for a [r, k] weight
    A = (torch.rand(r, k, generator=g) * 2 - 1) * bound if r else None
    B = torch.randn(n, r, generator=g) * 0.01 if r else None
    x = _bf16(torch.randn(m, k, generator=g))
    dy = _bf16(torch.randn(m, n, generator=g))
    return st, Nf4WeightCRef(packed, qs), w_deq, A, B, x, dy


@pytest.mark.parametrize("m,n,k,r", [(512, 256, 512, 16), (200, 512, 256, 16), (130, 128, 128, 32),
                                     (384, 1024, 640, 64), (256, 320, 256, 0)])
@pytest.mark.parametrize("variant", ["1cta", "2cta", "fused"])
def test_qlora_forward_backward(cuda_dev, m, n, k, r, variant, monkeypatch):
    """QLoRA forward and backward on the dequant + bf16 GEMM paths (one-CTA
    and pair kernels) and with the NF4 decode inside the GEMM ("fused"; shapes
    it does not take fall back to the dequant path)."""
    if variant == "fused":
        monkeypatch.setenv("FITQ_NF4_FUSED", "1")
    else:
        monkeypatch.setenv("FITQ_NF4_FUSED", "0")
        monkeypatch.setenv("FITQ_GEMM_VARIANT", variant)
    from fitllm_b200 import ops
    s = 2.0
    st, wref, w_deq, A, B, x, dy = _qlora_case(m, n, k, r, 7 + m, cuda_dev)
    xd, dyd = x.to(cuda_dev), dy.to(cuda_dev)
    Ad = A.to(cuda_dev) if r else None
    Bd = B.to(cuda_dev) if r else None
    y, t = ops.qlora_forward(xd, wref, Ad, Bd, s, want_t=True)
    Anp = A.numpy() if r else np.zeros((0, k), np.float32)
    Bnp = B.numpy() if r else np.zeros((n, 0), np.float32)
    ref = onf4.qlora_forward(x.float().numpy(), w_deq, Anp, Bnp, s)
    assert onf4.rel_err(y.float().cpu().numpy(), ref) < REL_TOL
    dx, ga, gb = ops.qlora_backward(xd, dyd, wref, Ad, Bd, s, t_saved=t)
    rdx, rda, rdb = onf4.qlora_backward(x.float().numpy(), w_deq, Anp, Bnp, s, dy.float().numpy())
    assert onf4.rel_err(dx.float().cpu().numpy(), rdx) < REL_TOL
    if r:
        assert onf4.rel_err(ga.cpu().numpy(), rda) < REL_TOL
        assert onf4.rel_err(gb.cpu().numpy(), rdb) < REL_TOL
        # recompute of T inside the backward gives the same grads
        dx2, ga2, gb2 = ops.qlora_backward(xd, dyd, wref, Ad, Bd, s, t_saved=None)
        assert onf4.rel_err(ga2.cpu().numpy(), rda) < REL_TOL
        assert onf4.rel_err(gb2.cpu().numpy(), rdb) < REL_TOL
    assert ops.device_status() == 0


@pytest.mark.parametrize("m", [1, 4, 16, 40, 64])
@pytest.mark.parametrize("n,k,r", [(256, 512, 16), (128, 1024, 0)])
def test_gemv_paths(cuda_dev, m, n, k, r):
    from fitllm_b200 import ops
    s = 2.0
    st, wref, w_deq, A, B, x, dy = _qlora_case(m, n, k, r, 31 + m, cuda_dev)
    Ad = A.to(cuda_dev) if r else None
    Bd = B.to(cuda_dev) if r else None
    bias = _bf16(torch.randn(n) * 0.1)
    y, _ = ops.qlora_forward(x.to(cuda_dev), wref, Ad, Bd, s, gemv=True, bias=bias.to(cuda_dev))
    Anp = A.numpy() if r else np.zeros((0, k), np.float32)
    Bnp = B.numpy() if r else np.zeros((n, 0), np.float32)
    ref = onf4.qlora_forward(x.float().numpy(), w_deq, Anp, Bnp, s) + bias.float().numpy()[None, :]
    assert onf4.rel_err(y.float().cpu().numpy(), ref) < REL_TOL
    # the GEMM path on the same inputs agrees too
    y2, _ = ops.qlora_forward(x.to(cuda_dev), wref, Ad, Bd, s, bias=bias.to(cuda_dev))
    assert onf4.rel_err(y2.float().cpu().numpy(), ref) < REL_TOL


@pytest.mark.parametrize("variant", ["default", "wide", "tc"])
@pytest.mark.parametrize("m,n,k,r,nested", [(1, 2048, 5120, 16, True), (3, 512, 27648, 0, True),
                                            (2, 1024, 5120, 16, True), (4, 2048, 1024, 0, False),
                                            (1, 6912, 5120, 0, True), (2, 1280, 27648, 0, True),
                                            (1, 640, 2048, 0, False), (4, 1536, 4096, 32, True),
                                            (8, 3072, 1024, 16, False), (5, 1024, 5120, 0, False),
                                            (1, 128, 256, 0, True), (16, 2048, 5120, 16, True),
                                            (40, 1024, 5120, 16, True), (64, 512, 1024, 0, False),
                                            (33, 384, 27648, 0, True), (48, 640, 5120, 16, False),
                                            (24, 1152, 1024, 0, True), (47, 256, 2048, 16, True)])
def test_gemv_decode_kernels(cuda_dev, monkeypatch, variant, m, n, k, r, nested):
    """The M <= 8 decode kernel, the tcgen05 skinny GEMM with the decoded
    weights in tensor memory (M <= 64; forced for M <= 8 by "tc") and the
    general skinny kernel ("wide"), on double-quantised and plain fp32 absmax
    weights, over several K slices, ring depths and token paddings."""
    monkeypatch.setenv("FITQ_GEMV_WIDE", "0" if variant == "default" else "1")
    monkeypatch.setenv("FITQ_GEMV_TC", {"default": "", "wide": "0", "tc": "1"}[variant])
    from fitllm_b200 import ops
    from fitllm_b200.nf4 import Nf4WeightCRef, QuantState
    s = 2.0
    st, wref, w_deq, A, B, x, dy = _qlora_case(m, n, k, r, 57 + m + n, cuda_dev)
    if not nested:  # same block scales, as fp32 absmax
        packed, _ = _state_to_device(st, cuda_dev)
        qs = QuantState(absmax=torch.from_numpy(onf4.absmax_decode(st).astype(np.float32)).to(cuda_dev),
                        shape=st.shape, quant_map=torch.from_numpy(st.quant_map.copy()).to(cuda_dev))
        wref = Nf4WeightCRef(packed, qs)
    Ad = A.to(cuda_dev) if r else None
    Bd = B.to(cuda_dev) if r else None
    y, _ = ops.qlora_forward(x.to(cuda_dev), wref, Ad, Bd, s, gemv=True)
    Anp = A.numpy() if r else np.zeros((0, k), np.float32)
    Bnp = B.numpy() if r else np.zeros((n, 0), np.float32)
    ref = onf4.qlora_forward(x.float().numpy(), w_deq, Anp, Bnp, s)
    assert onf4.rel_err(y.float().cpu().numpy(), ref) < REL_TOL
    assert ops.device_status() == 0


@pytest.mark.parametrize("m,n,k,r", [(1, 2048, 5120, 16), (4, 1024, 27648, 0), (8, 512, 1024, 32),
                                     (2, 5120, 5120, 16), (1, 6912, 5120, 0)])
def test_gemv_decode_deterministic(cuda_dev, monkeypatch, m, n, k, r):
    """The decode path (GEMV, LoRA T and finishing launches) gives the same
    bits on three calls over one reused workspace, within the 1e-2 contract of
    the oracle, and returns T when asked."""
    monkeypatch.setenv("FITQ_GEMV_WIDE", "0")
    from fitllm_b200 import _lib
    L = _lib.load()
    st, wref, w_deq, A, B, x, dy = _qlora_case(m, n, k, r, 91 + m, cuda_dev)
    Ad = A.to(cuda_dev).contiguous() if r else None
    Bd = B.to(cuda_dev).contiguous() if r else None
    xd = x.to(cuda_dev)
    nbytes = L.fitq_qlora_fwd_workspace(m, n, k, r)
    ws = torch.full((max(nbytes, 1),), 0x5A, dtype=torch.uint8, device=cuda_dev)  # not zeroed
    outs, ts = [], []
    for _ in range(3):
        y = torch.empty(m, n, dtype=torch.bfloat16, device=cuda_dev)
        t = torch.empty(m, max(r, 1), dtype=torch.bfloat16, device=cuda_dev)
        rc = L.fitq_qlora_fwd(wref.ref, xd.data_ptr(), m, _lib.ptr(Ad), _lib.ptr(Bd), r, 2.0, None,
                              y.data_ptr(), None, t.data_ptr() if r else None, ws.data_ptr(),
                              nbytes, torch.cuda.current_stream().cuda_stream)
        assert rc == 0, L.fitq_last_error()
        torch.cuda.synchronize()
        outs.append(y.clone())
        ts.append(t.clone())
    assert all(torch.equal(outs[0], o) for o in outs[1:])
    Anp = A.numpy() if r else np.zeros((0, k), np.float32)
    Bnp = B.numpy() if r else np.zeros((n, 0), np.float32)
    ref = onf4.qlora_forward(x.float().numpy(), w_deq, Anp, Bnp, 2.0)
    assert onf4.rel_err(outs[0].float().cpu().numpy(), ref) < REL_TOL
    if r:
        assert all(torch.equal(ts[0], t) for t in ts[1:])
        t_ref = x.float().numpy() @ A.bfloat16().float().numpy().T
        assert onf4.rel_err(ts[0].float().cpu().numpy(), t_ref) < REL_TOL


def _verify_attention_ref(q, kc, vc, prefix):
    """fp32 torch restatement: token i of q [B, T, H, D] attends to cache
    positions <= prefix + i; GQA heads h -> kv head h // (H / KVH)."""
    b, t, h, d = q.shape
    kvh = kc.shape[1]
    L = prefix + t
    k = kc[:, :, :L].float().repeat_interleave(h // kvh, dim=1)
    v = vc[:, :, :L].float().repeat_interleave(h // kvh, dim=1)
    s = torch.einsum("bthd,bhld->bhtl", q.float(), k) / math.sqrt(d)
    pos = torch.arange(L, device=q.device)
    lim = prefix + torch.arange(t, device=q.device)
    s = s.masked_fill(pos[None, None, None, :] > lim[None, None, :, None], float("-inf"))
    return torch.einsum("bhtl,bhld->bthd", torch.softmax(s, dim=-1), v)


@pytest.mark.parametrize("b,h,kvh,t,prefix,cap", [(8, 40, 8, 5, 4096, 4101), (2, 8, 2, 5, 300, 320),
                                                   (1, 8, 1, 4, 0, 4), (3, 4, 4, 1, 1000, 1001),
                                                   (1, 16, 1, 2, 4095, 5000), (2, 10, 2, 6, 63, 69)])
def test_verify_attention(cuda_dev, b, h, kvh, t, prefix, cap):
    """fitq_verify_attention against an fp32 softmax reference: GQA row
    folding (up to 32 rows), the prefix + causal mask, tile edges (prefix + T
    not a multiple of 64), a capacity beyond the valid length, one split
    (prefix 0) and many; within 1e-2 of the reference's norm."""
    from fitllm_b200 import ops
    g = torch.Generator(device=cuda_dev).manual_seed(b * 100 + h + t)
    q = torch.randn(b, t, h, 128, generator=g, device=cuda_dev).bfloat16()
    kc = torch.randn(b, kvh, cap, 128, generator=g, device=cuda_dev).bfloat16()
    vc = torch.randn(b, kvh, cap, 128, generator=g, device=cuda_dev).bfloat16()
    out = ops.verify_attention(q, kc, vc, prefix)
    ref = _verify_attention_ref(q, kc, vc, prefix)
    err = float((out.float() - ref).norm() / ref.norm())
    assert err < 1e-2, err
    assert ops.device_status() == 0
    # deterministic: a second call gives the same bits
    assert torch.equal(out, ops.verify_attention(q, kc, vc, prefix))


@pytest.mark.parametrize("rows,vocab,ignored", [(64, 4096, 0), (130, 152064, 7), (33, 1000, 33)])
def test_cross_entropy(cuda_dev, rows, vocab, ignored):
    """fitq_cross_entropy against torch's CrossEntropyLoss (mean over labels
    != -100) on the same bf16 logits: the loss, and the in-place
    d(scale * loss)/dlogits within 1e-2; a batch with every label ignored
    gives loss 0 and zero gradient."""
    from fitllm_b200 import _lib, ops
    import torch.nn.functional as F
    g = torch.Generator(device=cuda_dev).manual_seed(rows + vocab)
    logits = (torch.randn(rows, vocab, generator=g, device=cuda_dev) * 2).bfloat16()
    labels = torch.randint(0, vocab, (rows,), generator=g, device=cuda_dev)
    labels[:ignored] = -100
    ref = logits.float().requires_grad_(True)
    scale = 0.25
    L = _lib.load()
    work = logits.clone()
    loss = torch.empty((), dtype=torch.float32, device=cuda_dev)
    nb = L.fitq_cross_entropy_workspace(rows)
    ws = torch.empty(nb, dtype=torch.uint8, device=cuda_dev)
    _lib.check(L.fitq_cross_entropy(work.data_ptr(), labels.data_ptr(), rows, vocab, -100, scale,
                                    loss.data_ptr(), ws.data_ptr(), nb,
                                    torch.cuda.current_stream().cuda_stream), "fitq_cross_entropy")
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    if ignored == rows:
        assert float(loss) == 0.0 and not work.float().abs().sum().item()
        return
    lref = F.cross_entropy(ref, labels, ignore_index=-100)
    (lref * scale).backward()
    assert abs(float(loss) - float(lref.detach())) <= 1e-2 * abs(float(lref.detach()))
    gref = ref.grad
    assert float((work.float() - gref).norm() / gref.norm()) < 1e-2


def test_lm_head_loss_and_grad(cuda_dev):
    """Final RMSNorm + lm_head + CE (fitllm_b200/lm_head.py) against an fp32
    autograd restatement of fitllm/backward.py:188-198: the mean loss of each
    micro-batch and grad of loss * (1 / grad_accum) w.r.t. h_last, within 1e-2."""
    import torch.nn.functional as F
    from fitllm_b200.lm_head import LMHeadLoss
    g = torch.Generator(device=cuda_dev).manual_seed(77)
    nmb, s, hid, vocab = 2, 64, 256, 4096
    h = torch.randn(nmb, s, hid, generator=g, device=cuda_dev).bfloat16()
    nw = (1 + 0.1 * torch.randn(hid, generator=g, device=cuda_dev)).bfloat16()
    w = (torch.randn(vocab, hid, generator=g, device=cuda_dev) * 0.05).bfloat16()
    labels = torch.randint(0, vocab, (nmb, s), generator=g, device=cuda_dev)
    labels[0, :10] = -100
    head = LMHeadLoss(nw, w, eps=1e-6)
    losses, grad = head.loss_and_grad_microbatches(h, labels, loss_scale=1.0 / nmb)
    for i in range(nmb):
        x = h[i].float().requires_grad_(True)
        y = nw.float() * (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6))
        loss = F.cross_entropy(y @ w.float().t(), labels[i], ignore_index=-100)
        (loss / nmb).backward()
        assert abs(float(losses[i]) - float(loss.detach())) <= 1e-2 * float(loss.detach())
        assert float((grad[i].float() - x.grad).norm() / x.grad.norm()) < 1e-2


@pytest.mark.parametrize("m,shapes,nested", [(40, [(512, 1024, 16), (128, 1024, 0), (128, 1024, 16)], True),
                                             (16, [(1024, 2048, 0), (1024, 2048, 0)], True),
                                             (64, [(384, 512, 0), (256, 512, 16)], False),
                                             (4, [(256, 512, 16), (128, 512, 0)], True),
                                             (1, [(1024, 5120, 16), (256, 5120, 0), (256, 5120, 16)], True),
                                             (2, [(2048, 1024, 0), (2048, 1024, 0)], False),
                                             (8, [(512, 1024, 32), (192, 1024, 0), (64, 1024, 16)], True)])
def test_gemv_grouped(cuda_dev, m, shapes, nested):
    """fitq_nf4_gemv_grouped: up to three projections of one x (one tcgen05
    launch over all their tiles for 8 < M <= 64, one decode-kernel launch for
    M <= 8) give
    each projection's fitq_nf4_gemv result within 1e-2 of the oracle, with
    LoRA, bias and y_add per job."""
    from fitllm_b200 import ops
    from fitllm_b200.nf4 import Nf4WeightCRef, QuantState
    g = torch.Generator(device=cuda_dev).manual_seed(m + len(shapes))
    k = shapes[0][1]
    x = torch.randn(m, k, generator=g, device=cuda_dev).bfloat16()
    jobs, refs = [], []
    for i, (n, kk, r) in enumerate(shapes):
        st, wref, w_deq, A, B, _, _ = _qlora_case(m, n, kk, r, 300 + i * 7 + m, cuda_dev)
        if not nested:
            packed, _ = _state_to_device(st, cuda_dev)
            qs = QuantState(absmax=torch.from_numpy(onf4.absmax_decode(st).astype(np.float32)).to(cuda_dev),
                            shape=st.shape, quant_map=torch.from_numpy(st.quant_map.copy()).to(cuda_dev))
            wref = Nf4WeightCRef(packed, qs)
        bias = (torch.randn(n, generator=g, device=cuda_dev) * 0.1).bfloat16()
        y_add = torch.randn(m, n, generator=g, device=cuda_dev).bfloat16() if i == 0 else None
        Ad = A.to(cuda_dev) if r else None
        Bd = B.to(cuda_dev) if r else None
        jobs.append((wref, Ad, Bd, 2.0, bias, y_add))
        Anp = A.numpy() if r else np.zeros((0, kk), np.float32)
        Bnp = B.numpy() if r else np.zeros((n, 0), np.float32)
        ref = onf4.qlora_forward(x.float().cpu().numpy(), w_deq, Anp, Bnp, 2.0) + bias.float().cpu().numpy()
        if y_add is not None:
            ref = ref + y_add.float().cpu().numpy()
        refs.append(ref)
    outs = ops.nf4_gemv_grouped(x, jobs)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    for y, ref in zip(outs, refs):
        assert onf4.rel_err(y.float().cpu().numpy(), ref) < REL_TOL
    # same results as the per-projection calls
    for (wref, Ad, Bd, s, bias, y_add), y in zip(jobs, outs):
        y1, _ = ops.qlora_forward(x, wref, Ad, Bd, s, gemv=True, bias=bias, y_add=y_add)
        assert float((y.float() - y1.float()).norm() / y1.float().norm()) < 1e-3


@pytest.mark.parametrize("m,n,k,bias", [(16, 1024, 2048, False), (40, 512, 1024, True), (64, 384, 512, False),
                                        (4, 256, 512, True)])
def test_gemv_swiglu(cuda_dev, m, n, k, bias):
    """fitq_nf4_gemv_swiglu (gate/up + SwiGLU in one grouped launch and one
    finishing pass for 8 < M <= 64, the per-projection calls + the SwiGLU
    kernel otherwise) is bit-identical to fitq_nf4_gemv_grouped followed by
    fitq_swiglu_fwd, and within 1e-2 of the oracle's SiLU(gate) * up."""
    from fitllm_b200 import ops
    from fitllm_b200.layer_ops import swiglu
    g = torch.Generator(device=cuda_dev).manual_seed(m + n)
    x = torch.randn(m, k, generator=g, device=cuda_dev).bfloat16()
    jobs, refs = [], []
    for i in range(2):
        _, wref, w_deq, _, _, _, _ = _qlora_case(m, n, k, 0, 500 + i * 11 + m, cuda_dev)
        b = (torch.randn(n, generator=g, device=cuda_dev) * 0.1).bfloat16() if bias else None
        jobs.append((wref, None, None, 1.0, b, None))
        ref = x.float().cpu().numpy() @ w_deq.T
        if b is not None:
            ref = ref + b.float().cpu().numpy()
        refs.append(ref)
    act = ops.nf4_gemv_swiglu(x, jobs[0], jobs[1])
    gate, up = ops.nf4_gemv_grouped(x, jobs)
    act2 = swiglu(gate, up)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    assert torch.equal(act, act2)
    ga, ua = refs
    ref = ga / (1.0 + np.exp(-ga)) * ua
    assert onf4.rel_err(act.float().cpu().numpy(), ref) < REL_TOL


def test_bounded_wait_timeout_leaves_context_usable(cuda_dev):
    """The failure path of the device waits, without a fault: a wait on an
    mbarrier that nothing completes runs out after its limit, records
    FITQ_ERR_TIMEOUT in the status word and returns; the context keeps
    working (a GEMM right after is correct) and the status clears."""
    from fitllm_b200 import _lib, ops
    L = _lib.load()
    assert ops.device_status(reset=True) == 0
    stream = torch.cuda.current_stream().cuda_stream
    assert L.fitq_selftest_wait_timeout(0, None, stream) == 1  # FITQ_ERR_ARG: limit out of range
    elapsed = torch.zeros(1, dtype=torch.int64, device=cuda_dev)
    limit = 20_000_000  # 20 ms
    assert L.fitq_selftest_wait_timeout(limit, elapsed.data_ptr(), stream) == 0
    assert ops.device_status(reset=True) == 7  # FITQ_ERR_TIMEOUT
    waited = int(elapsed.item())
    assert limit <= waited < 1_000_000_000
    assert ops.device_status() == 0
    g = torch.Generator(device="cpu").manual_seed(3)
    a = _bf16(torch.randn(256, 512, generator=g)).to(cuda_dev)
    b = _bf16(torch.randn(128, 512, generator=g)).to(cuda_dev)
    c = ops.gemm_bf16_tn(a, b)
    assert onf4.rel_err(c.float().cpu().numpy(), (a.float() @ b.float().T).cpu().numpy()) < 4e-3
    assert ops.device_status() == 0


def test_side_stream_off_gives_same_bits(cuda_dev, tmp_path):
    """The QLoRA GEMM path with its weight side on the caller's stream
    (FITQ_SIDE_STREAM=0, read once per process, so run in a child process)
    returns the same bits as with the forked side stream."""
    import subprocess
    import sys
    script = tmp_path / "side.py"
    out = tmp_path / "out_{}.pt"
    script.write_text(
        "import sys, torch\n"
        "sys.path.insert(0, %r)\n"
        "from fitllm_b200 import ops\n"
        "from fitllm_b200.qlora import Linear4bit\n"
        "dev = torch.device('cuda', 0)\n"
        "g = torch.Generator(device=dev).manual_seed(3)\n"
        "w = Linear4bit.from_float(torch.randn(1024, 768, generator=g, device=dev) * 0.02, None).wref()\n"
        "x = torch.randn(300, 768, generator=g, device=dev).bfloat16()\n"
        "dy = torch.randn(300, 1024, generator=g, device=dev).bfloat16()\n"
        "A = torch.randn(16, 768, generator=g, device=dev) * 0.02\n"
        "B = torch.randn(1024, 16, generator=g, device=dev) * 0.02\n"
        "y, t = ops.qlora_forward(x, w, A, B, 2.0, want_t=True)\n"
        "dx, ga, gb = ops.qlora_backward(x, dy, w, A, B, 2.0, t_saved=t)\n"
        "torch.cuda.synchronize()\n"
        "torch.save([v.cpu() for v in (y, t, dx, ga, gb)], sys.argv[1])\n" % str(__import__('pathlib').Path(__file__).resolve().parents[1]))
    import os
    res = []
    for side in ("1", "0"):
        env = dict(os.environ, FITQ_SIDE_STREAM=side, FITQ_NF4_FUSED="0")
        path = str(out).format(side)
        subprocess.run([sys.executable, str(script), path], check=True, env=env, timeout=300)
        res.append(torch.load(path))
    for a, b in zip(*res):
        assert torch.equal(a, b)
