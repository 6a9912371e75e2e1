"""fitq_nf4_gemv_noalloc: the decode GEMV for callers that cannot allocate.

Some hosts drive the decode step through the C ABI without any CUDA
allocator of their own (a foreign-language runtime, or one that must budget
every device allocation in advance), so they cannot hand fitq_nf4_gemv the
scratch workspace it asks for.  The no-allocation variant takes its scratch
from a fixed array inside the library.  These tests call it through the C ABI
and check it against the workspace-taking entry point on two calls in a row
(the shared scratch keeps the previous call's contents, which must not leak
into the next result), within the 1e-2 relative tolerance the other kernel
tests use, and check that a shape needing more than the fixed scratch is
rejected.  This file is collected last on purpose.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import nf4 as onf4

pytestmark = pytest.mark.gpu
REL = 1e-2


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
    return Nf4WeightCRef(packed, qs)


def _call_noalloc(L, w, x, a, b, rank, scale, bias, y):
    p = lambda t: None if t is None else t.data_ptr()
    return L.fitq_nf4_gemv_noalloc(w.ref, x.data_ptr(), x.shape[0], p(a), p(b), rank, scale,
                                   p(bias), y.data_ptr(), None,
                                   torch.cuda.current_stream().cuda_stream)


def _call_workspace(L, w, x, a, b, rank, scale, bias, y):
    p = lambda t: None if t is None else t.data_ptr()
    n, k = w.c.n_out, w.c.k_in
    nbytes = L.fitq_nf4_gemv_workspace(x.shape[0], n, k, rank)
    ws = torch.zeros(max(nbytes, 1), dtype=torch.uint8, device=x.device)  # zero counter prefix
    rc = L.fitq_nf4_gemv(w.ref, x.data_ptr(), x.shape[0], p(a), p(b), rank, scale, p(bias),
                         y.data_ptr(), None, ws.data_ptr(), nbytes,
                         torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return rc


@pytest.mark.parametrize("m,n,k,rank", [(1, 512, 1024, 16), (40, 1024, 512, 16), (16, 256, 2048, 0)])
def test_noalloc_matches_workspace_gemv_two_calls(cuda_dev, m, n, k, rank):
    from fitllm_b200 import _lib
    L = _lib.load()
    w = _weight(n, k, 100 + m, cuda_dev)
    g = torch.Generator().manual_seed(7 + m)
    for call in range(2):  # second call sees the scratch left by the first
        x = torch.randn(m, k, generator=g).bfloat16().to(cuda_dev)
        a = ((torch.rand(rank, k, generator=g) * 2 - 1) / np.sqrt(k)).to(cuda_dev) if rank else None
        b = (torch.randn(n, rank, generator=g) * 0.02).to(cuda_dev) if rank else None
        bias = (torch.randn(n, generator=g) * 0.1).bfloat16().to(cuda_dev)
        y0 = torch.empty(m, n, dtype=torch.bfloat16, device=cuda_dev)
        y1 = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=cuda_dev)
        assert _call_workspace(L, w, x, a, b, rank, 2.0, bias, y0) == 0
        rc = _call_noalloc(L, w, x, a, b, rank, 2.0, bias, y1)
        assert rc == 0, L.fitq_last_error()
        torch.cuda.synchronize()
        assert onf4.rel_err(y1.float().cpu().numpy(), y0.float().cpu().numpy()) < REL, call
        assert torch.isfinite(y1.float()).all()


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
    assert rc == 5  # FITQ_ERR_WORKSPACE
    assert b"scratch" in L.fitq_last_error()
