"""C-ABI calls from a host thread that has made no CUDA call yet.

Such a thread has no current CUDA context.  PyTorch's autograd worker for
device 0 is one: the backward of a layer runs there, so the first backward
projection of a FitLLM layer step (down_proj's input gradient) is issued from
it, and so is any call a foreign host makes from a thread of its own.  The
runtime binds the context for kernel launches by itself, but the driver's
tensor-map encoding the tcgen05 GEMMs need does not, and some drivers refuse
it there.  These tests issue the GEMM entry points from a fresh thread, with
every buffer allocated beforehand on the main thread and nothing but the C
call in the thread, and require the same bits as the same calls made from the
main thread.
"""
import threading

import pytest
import torch

pytestmark = pytest.mark.gpu


def _calls(L, w, x, dy, y, dx, ws_f, nf, ws_b, nb, stream):
    """Forward y = x.W^T and input gradient dx = dy.W through the C ABI, no
    LoRA (so no launch precedes the GEMM's own set-up); returns both codes."""
    rf = L.fitq_qlora_fwd(w.ref, x.data_ptr(), x.shape[0], None, None, 0, 1.0, None, y.data_ptr(),
                          None, None, ws_f.data_ptr(), nf, stream)
    rb = L.fitq_qlora_bwd(w.ref, None, dy.data_ptr(), dy.shape[0], None, None, 0, 1.0, None,
                          dx.data_ptr(), 0, None, None, 0, ws_b.data_ptr(), nb, stream)
    return rf, rb


@pytest.mark.parametrize("fused", ["1", "0"])
def test_gemm_entry_points_from_a_fresh_host_thread(cuda_dev, monkeypatch, fused):
    from fitllm_b200 import _lib
    from fitllm_b200.qlora import Linear4bit
    monkeypatch.setenv("FITQ_NF4_FUSED", fused)  # NF4 decoded in the GEMM, or dequant + GEMM
    L = _lib.load()
    m, n, k = 256, 1024, 768
    g = torch.Generator(device=cuda_dev).manual_seed(31)
    w = Linear4bit.from_float(torch.randn(n, k, generator=g, device=cuda_dev) * 0.02, None).wref()
    x = torch.randn(m, k, generator=g, device=cuda_dev).bfloat16()
    dy = torch.randn(m, n, generator=g, device=cuda_dev).bfloat16()
    nf, nb = L.fitq_qlora_fwd_workspace(m, n, k, 0), L.fitq_qlora_bwd_workspace(m, n, k, 0)
    ws_f = torch.empty(max(nf, 1), dtype=torch.uint8, device=cuda_dev)
    ws_b = torch.empty(max(nb, 1), dtype=torch.uint8, device=cuda_dev)
    y0, y1 = (torch.empty(m, n, dtype=torch.bfloat16, device=cuda_dev) for _ in range(2))
    dx0, dx1 = (torch.empty(m, k, dtype=torch.bfloat16, device=cuda_dev) for _ in range(2))
    stream = torch.cuda.current_stream().cuda_stream
    assert _calls(L, w, x, dy, y0, dx0, ws_f, nf, ws_b, nb, stream) == (0, 0), L.fitq_last_error()
    torch.cuda.synchronize()

    out = {}

    def worker():
        out["rc"] = _calls(L, w, x, dy, y1, dx1, ws_f, nf, ws_b, nb, stream)
        out["err"] = L.fitq_last_error()

    th = threading.Thread(target=worker)
    th.start()
    th.join(timeout=120)
    assert not th.is_alive()
    assert out["rc"] == (0, 0), out["err"]
    torch.cuda.synchronize()
    assert torch.equal(y1, y0)
    assert torch.equal(dx1, dx0)
