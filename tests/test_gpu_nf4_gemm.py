"""The NF4 GEMM with the dequant fused into the tcgen05 producer path.

* Bit-exactness of the decoded operand: with x = I the forward computes
  I . W_deq^T = W_deq^T and with dY = I the input-gradient GEMM computes
  I . W_deq = W_deq; one product per output element, accumulated in fp32 and
  rounded to bf16, reproduces the decoded weight exactly.  So the outputs must
  equal the oracle's bitsandbytes dequant bit for bit -- for the K-major
  (forward) and MN-major (dX) operand layouts, on the CTA-pair kernel (256-
  and 512-row tiles) and the one-CTA kernel, double-quantised and plain fp32
  absmax, one tile and many tiles per CTA.
* The full QLoRA forward / backward through the fused GEMM (LoRA K-block,
  bias, residual add, M not a multiple of the 256-row tile) against the
  oracle within the 1e-2 contract, and against the dequant + bf16 GEMM path.
"""
import numpy as np
import pytest
import torch

from oracle import nf4 as onf4

pytestmark = pytest.mark.gpu
REL = 1e-2


def _weight(n, k, seed, dev, nested=True):
    from fitllm_b200.nf4 import Nf4WeightCRef, QuantState
    g = torch.Generator().manual_seed(seed)
    st = onf4.quantize((torch.randn(n, k, generator=g) * 0.02).numpy())
    packed = torch.from_numpy(st.packed.copy()).to(dev)
    if nested:
        qs = QuantState(absmax=torch.from_numpy(st.absmax_code.copy()).to(dev), shape=(n, k),
                        quant_map=torch.from_numpy(st.quant_map.copy()).to(dev),
                        nested_absmax=torch.from_numpy(st.nested_absmax.copy()).to(dev),
                        nested_quant_map=torch.from_numpy(st.nested_quant_map.copy()).to(dev),
                        offset=float(st.offset))
    else:
        qs = QuantState(absmax=torch.from_numpy(onf4.absmax_decode(st).astype(np.float32)).to(dev),
                        shape=(n, k), quant_map=torch.from_numpy(st.quant_map.copy()).to(dev))
    return st, Nf4WeightCRef(packed, qs)


KERNELS = ["pair256", "pair512", "1cta"]


def _set_kernel(monkeypatch, kernel):
    """pair256 / pair512: the CTA-pair kernel with 256- or 512-row tiles where
    the output columns are a multiple of 256 (the one-CTA kernel otherwise);
    1cta: the one-CTA kernel throughout."""
    if kernel == "1cta":
        monkeypatch.setenv("FITQ_NF4_GEMM", "1cta")
    else:
        monkeypatch.setenv("FITQ_NF4_MSUB", "2" if kernel == "pair512" else "1")


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("n,k,nested", [(128, 64, True), (384, 512, True), (256, 1024, False),
                                        (1024, 2048, True), (640, 1280, False)])
def test_fused_decode_bit_exact(cuda_dev, monkeypatch, n, k, nested, kernel):
    monkeypatch.setenv("FITQ_NF4_FUSED", "1")
    _set_kernel(monkeypatch, kernel)
    from fitllm_b200 import ops
    st, wref = _weight(n, k, 900 + n + k, cuda_dev, nested)
    ref = onf4.dequant(st, "bf16")  # uint16 bits [n, k]
    eye_k = torch.eye(k, dtype=torch.bfloat16, device=cuda_dev)
    y, _ = ops.qlora_forward(eye_k, wref, None, None, 1.0)  # [k, n] = W^T
    got = y.view(torch.int16).cpu().numpy().view(np.uint16)
    assert np.array_equal(got, ref.T)
    eye_n = torch.eye(n, dtype=torch.bfloat16, device=cuda_dev)
    dx, _, _ = ops.qlora_backward(None, eye_n, wref, None, None, 1.0)  # [n, k] = W
    got = dx.view(torch.int16).cpu().numpy().view(np.uint16)
    assert np.array_equal(got, ref)
    assert ops.device_status() == 0


@pytest.mark.parametrize("kernel", KERNELS)
@pytest.mark.parametrize("m,n,k,r,nested", [(1000, 384, 640, 16, True), (300, 1280, 5120, 16, True),
                                            (2048, 1024, 1024, 32, False), (777, 256, 2048, 0, True),
                                            (4096, 512, 512, 64, True), (5000, 2048, 1536, 16, True)])
def test_fused_qlora_vs_oracle_and_dequant_path(cuda_dev, monkeypatch, m, n, k, r, nested, kernel):
    _set_kernel(monkeypatch, kernel)
    from fitllm_b200 import ops
    s = 2.0
    st, wref = _weight(n, k, 950 + m, cuda_dev, nested)
    w_deq = onf4.bf16_bits_to_f32(onf4.dequant(st, "bf16"))
    g = torch.Generator().manual_seed(m + n)
    A = ((torch.rand(r, k, generator=g) * 2 - 1) / np.sqrt(k)) if r else None
    B = (torch.randn(n, r, generator=g) * 0.01) if r else None
    x = torch.randn(m, k, generator=g).bfloat16()
    dy = torch.randn(m, n, generator=g).bfloat16()
    bias = (torch.randn(n, generator=g) * 0.1).bfloat16()
    y_add = torch.randn(m, n, generator=g).bfloat16()
    dx0 = torch.randn(m, k, generator=g).bfloat16()
    Ad = A.to(cuda_dev) if r else None
    Bd = B.to(cuda_dev) if r else None
    outs = {}
    for fused in ("1", "0"):
        monkeypatch.setenv("FITQ_NF4_FUSED", fused)
        xd, dyd = x.to(cuda_dev), dy.to(cuda_dev)
        y, t = ops.qlora_forward(xd, wref, Ad, Bd, s, want_t=bool(r), bias=bias.to(cuda_dev),
                                 y_add=y_add.to(cuda_dev))
        dx = dx0.to(cuda_dev).clone()  # accumulated into
        _, ga, gb = ops.qlora_backward(xd, dyd, wref, Ad, Bd, s, t_saved=t, dx=dx)
        torch.cuda.synchronize()
        assert ops.device_status() == 0
        outs[fused] = (y.float().cpu().numpy(), dx.float().cpu().numpy(),
                       None if ga is None else ga.cpu().numpy(), None if gb is None else gb.cpu().numpy())
    Anp = A.numpy() if r else np.zeros((0, k), np.float32)
    Bnp = B.numpy() if r else np.zeros((n, 0), np.float32)
    ry = onf4.qlora_forward(x.float().numpy(), w_deq, Anp, Bnp, s) + bias.float().numpy() + y_add.float().numpy()
    rdx, _, _ = onf4.qlora_backward(x.float().numpy(), w_deq, Anp, Bnp, s, dy.float().numpy())
    rdx = rdx + dx0.float().numpy()
    y1, dx1 = outs["1"][0], outs["1"][1]
    assert onf4.rel_err(y1, ry) < REL
    assert onf4.rel_err(dx1, rdx) < REL
    # same arithmetic as the dequant + bf16 GEMM path up to accumulation order
    assert onf4.rel_err(y1, outs["0"][0]) < 2e-3
    assert onf4.rel_err(dx1, outs["0"][1]) < 2e-3
