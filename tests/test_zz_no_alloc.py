"""fitq_nf4_gemv_noalloc: the decode GEMV for callers that cannot allocate.

Some hosts drive the decode step through the C ABI without any CUDA
allocator of their own (a foreign-language runtime, or one that must budget
every device allocation in advance), so they cannot hand fitq_nf4_gemv the
scratch workspace it asks for.  The no-allocation variant takes its scratch
from a fixed array inside the library and otherwise runs fitq_nf4_gemv's
checks, kernel choice and arithmetic.  These tests call it through the C ABI
on two calls in a row (the shared scratch keeps the previous call's
contents, which must not leak into the next result) and check it against the
workspace-taking entry point (bit-identical) and against the oracle (within
the 1e-2 relative tolerance of the other kernel tests); that a shape needing
more than the fixed scratch is rejected; and that a misaligned LoRA pointer
is refused on the host before anything is launched.  This file is collected
last on purpose.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import nf4 as onf4

pytestmark = pytest.mark.gpu
REL = 1e-2
FITQ_ERR_ALIGN = 3
FITQ_ERR_WORKSPACE = 5


def _weight(n, k, seed, dev):
    from fitllm_b200.nf4 import Nf4WeightCRef, QuantState
    g = torch.Generator().manual_seed(seed)
    st = onf4.quantize((torch.randn(n, k, generator=g) * 0.02).numpy())
    packed = torch.from_numpy(st.packed.copy()).to(dev)
    qs = QuantState(absmax=torch.from_numpy(st.absmax_code.copy()).to(dev), shape=(n, k),
                    quant_map=torch.from_numpy(st.quant_map.copy()).to(dev),
                    nested_absmax=torch.from_numpy(st.nested_absmax.copy()).to(dev),
                    nested_quant_map=torch.from_numpy(st.nested_quant_map.copy()).to(dev),
                    offset=float(st.offset))
    return Nf4WeightCRef(packed, qs), onf4.bf16_bits_to_f32(onf4.dequant(st, "bf16"))


def _call_noalloc(L, w, x, a, b, rank, scale, bias, y):
    p = lambda t: None if t is None else t.data_ptr()
    return L.fitq_nf4_gemv_noalloc(w.ref, x.data_ptr(), x.shape[0], p(a), p(b), rank, scale,
                                   p(bias), y.data_ptr(), None,
                                   torch.cuda.current_stream().cuda_stream)


def _call_workspace(L, w, x, a, b, rank, scale, bias, y):
    p = lambda t: None if t is None else t.data_ptr()
    n, k = w.c.n_out, w.c.k_in
    nbytes = L.fitq_nf4_gemv_workspace(x.shape[0], n, k, rank)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=x.device)
    rc = L.fitq_nf4_gemv(w.ref, x.data_ptr(), x.shape[0], p(a), p(b), rank, scale, p(bias),
                         y.data_ptr(), None, ws.data_ptr(), nbytes,
                         torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return rc


# decode kernel (M <= 8): one K slice with and without LoRA, several slices
# (K = 5120 and 27648); tcgen05 skinny GEMM (8 < M <= 64) with and without LoRA
@pytest.mark.parametrize("m,n,k,rank", [(1, 512, 1024, 16), (4, 2048, 5120, 16), (3, 1024, 27648, 0),
                                        (8, 384, 1280, 16), (40, 1024, 512, 16), (16, 256, 2048, 0)])
def test_noalloc_matches_workspace_gemv_two_calls(cuda_dev, m, n, k, rank):
    from fitllm_b200 import _lib
    L = _lib.load()
    w, w_deq = _weight(n, k, 100 + m, cuda_dev)
    g = torch.Generator().manual_seed(7 + m)
    for call in range(2):  # second call sees the scratch left by the first
        x = torch.randn(m, k, generator=g).bfloat16()
        a = ((torch.rand(rank, k, generator=g) * 2 - 1) / np.sqrt(k)) if rank else None
        b = (torch.randn(n, rank, generator=g) * 0.02) if rank else None
        bias = (torch.randn(n, generator=g) * 0.1).bfloat16()
        xd, biasd = x.to(cuda_dev), bias.to(cuda_dev)
        ad = a.to(cuda_dev) if rank else None
        bd = b.to(cuda_dev) if rank else None
        y0 = torch.empty(m, n, dtype=torch.bfloat16, device=cuda_dev)
        y1 = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=cuda_dev)
        assert _call_workspace(L, w, xd, ad, bd, rank, 2.0, biasd, y0) == 0
        rc = _call_noalloc(L, w, xd, ad, bd, rank, 2.0, biasd, y1)
        assert rc == 0, L.fitq_last_error()
        torch.cuda.synchronize()
        assert torch.equal(y1, y0), call  # same kernels, same arithmetic
        A = a.numpy() if rank else np.zeros((0, k), np.float32)
        B = b.numpy() if rank else np.zeros((n, 0), np.float32)
        ref = onf4.qlora_forward(x.float().numpy(), w_deq, A, B, 2.0) + bias.float().numpy()
        assert onf4.rel_err(y1.float().cpu().numpy(), ref) < REL, call


def test_noalloc_rejects_shapes_beyond_its_scratch(cuda_dev):
    from fitllm_b200 import _lib
    L = _lib.load()
    n, k, m = 65536, 256, 64  # 64 x 65536 fp32 partial products alone exceed 8 MiB
    packed = torch.zeros(n * k // 2, dtype=torch.uint8, device=cuda_dev)
    absmax = torch.ones(n * k // 64, dtype=torch.float32, device=cuda_dev)
    qm = torch.tensor(onf4.NF4_LEVELS, device=cuda_dev)
    from fitllm_b200._lib import Nf4WeightC
    wc = Nf4WeightC(packed=packed.data_ptr(), absmax_f32=absmax.data_ptr(), quant_map=qm.data_ptr(),
                    n_out=n, k_in=k)
    x = torch.zeros(m, k, dtype=torch.bfloat16, device=cuda_dev)
    y = torch.zeros(m, n, dtype=torch.bfloat16, device=cuda_dev)
    rc = L.fitq_nf4_gemv_noalloc(ctypes.byref(wc), x.data_ptr(), m, None, None, 0, 1.0, None,
                                 y.data_ptr(), None, torch.cuda.current_stream().cuda_stream)
    assert rc == FITQ_ERR_WORKSPACE
    assert b"scratch" in L.fitq_last_error()


@pytest.mark.parametrize("which", ["lora_a", "lora_b"])
def test_noalloc_refuses_misaligned_lora_pointer(cuda_dev, which):
    """The LoRA kernels read A and B with 16-byte loads: a pointer off the
    16-byte grid is refused with FITQ_ERR_ALIGN on the host, nothing launched."""
    from fitllm_b200 import _lib
    L = _lib.load()
    m, n, k, rank = 1, 256, 512, 16
    w, _ = _weight(n, k, 5, cuda_dev)
    x = torch.randn(m, k, device=cuda_dev).bfloat16()
    a = torch.randn(rank * k + 4, device=cuda_dev)
    b = torch.randn(n * rank + 4, device=cuda_dev)
    pa = a.data_ptr() + (4 if which == "lora_a" else 0)
    pb = b.data_ptr() + (4 if which == "lora_b" else 0)
    y = torch.zeros(m, n, dtype=torch.bfloat16, device=cuda_dev)
    torch.cuda.synchronize()
    before = L.fitq_launch_count()
    rc = L.fitq_nf4_gemv_noalloc(w.ref, x.data_ptr(), m, pa, pb, rank, 2.0, None, y.data_ptr(),
                                 None, torch.cuda.current_stream().cuda_stream)
    assert rc == FITQ_ERR_ALIGN
    assert L.fitq_launch_count() == before
    assert not y.any()
