"""Caller-owned workspaces: the result does not depend on what the workspace
held before the call, and nothing is written past the size the workspace
query returned.

Every projection, attention and reduction call of the library takes its
scratch (dequantised weights, padded LoRA operands, split-K partials) from one
caller-provided buffer of fitq_*_workspace() bytes.  Here that buffer is the
head of a larger allocation whose tail is a guard band; the buffer and the
guard are filled with 0x00, 0xFF and 0x5A before each call.  The outputs must
be bit-identical for every fill and the guard must come back untouched.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

GUARD = 4096
FILLS = (0x00, 0xFF, 0x5A)

# (M, N, K, rank): split and unsplit LoRA projections, the decode and
# tcgen05 skinny GEMV paths, N != K, ranks 16-64
SHAPES = [(128, 256, 256, 16), (128, 128, 256, 16), (100, 1024, 5120, 32), (512, 1024, 1024, 64),
          (5000, 1024, 1024, 16), (20, 1024, 5120, 16), (2, 1024, 5120, 16)]


@pytest.fixture
def guarded_workspace(monkeypatch):
    from fitllm_b200 import ops
    state = {"fill": 0, "bufs": []}

    def _ws(nbytes, dev):
        n = max(int(nbytes), 1)
        big = torch.full((n + GUARD,), state["fill"], dtype=torch.uint8, device=dev)
        state["bufs"].append((big, n))
        return big[:n]

    monkeypatch.setattr(ops, "_workspace", _ws)
    return state


def _check_guards(state):
    torch.cuda.synchronize()
    for big, n in state["bufs"]:
        tail = big[n:]
        assert bool((tail == state["fill"]).all()), f"write past the {n}-byte workspace"
    state["bufs"].clear()


@pytest.mark.parametrize("m,n,k,r", SHAPES)
def test_qlora_workspace_contents_and_bounds(cuda_dev, guarded_workspace, m, n, k, r):
    from fitllm_b200 import ops
    from fitllm_b200.qlora import Linear4bit
    g = torch.Generator(device=cuda_dev).manual_seed(m + n + r)
    w = Linear4bit.from_float(torch.randn(n, k, generator=g, device=cuda_dev) * 0.02, None).wref()
    a = (torch.randn(r, k, generator=g, device=cuda_dev) * 0.02).contiguous()
    b = (torch.randn(n, r, generator=g, device=cuda_dev) * 0.02).contiguous()
    x = torch.randn(m, k, generator=g, device=cuda_dev).bfloat16()
    dy = torch.randn(m, n, generator=g, device=cuda_dev).bfloat16()
    ref = None
    for fill in FILLS:
        guarded_workspace["fill"] = fill
        y, t = ops.qlora_forward(x, w, a, b, 2.0, want_t=True)
        y0, _ = ops.qlora_forward(x, w, a, b, 2.0)
        dx, da, db = ops.qlora_backward(x, dy, w, a, b, 2.0)
        dx2, da2, db2 = ops.qlora_backward(x, dy, w, a, b, 2.0, t_saved=t)
        _check_guards(guarded_workspace)
        assert ops.device_status() == 0
        out = [y, y0, t, dx, da, db, dx2, da2, db2]
        if ref is None:
            ref = [o.clone() for o in out]
            assert torch.equal(y, y0)
            assert torch.equal(dx, dx2) and torch.equal(da, da2) and torch.equal(db, db2)
            continue
        for i, (o, e) in enumerate(zip(out, ref)):
            assert torch.equal(o, e), f"output {i} changed with workspace fill {fill:#x}"


@pytest.mark.parametrize("m", [1, 4, 40])
def test_grouped_gemv_workspace_contents_and_bounds(cuda_dev, guarded_workspace, m):
    from fitllm_b200.qlora import Linear4bit, QLoRALinear4bit, grouped_forward
    g = torch.Generator(device=cuda_dev).manual_seed(m)
    mods = []
    for n in (1024, 256, 256):
        base = Linear4bit.from_float(torch.randn(n, 1024, generator=g, device=cuda_dev) * 0.02, None)
        mod = QLoRALinear4bit(base, r=16, lora_alpha=32.0).to(cuda_dev)
        with torch.no_grad():
            mod.lora_B["default"].weight.normal_(0.0, 0.02, generator=g)
        mods.append(mod)
    x = torch.randn(m, 1024, generator=g, device=cuda_dev).bfloat16()
    ref = None
    for fill in FILLS:
        guarded_workspace["fill"] = fill
        with torch.no_grad():
            ys = grouped_forward(mods, x)
        _check_guards(guarded_workspace)
        if ref is None:
            ref = [y.clone() for y in ys]
            continue
        for y, e in zip(ys, ref):
            assert torch.equal(y, e)


def _nf4(n, k, seed, dev):
    from fitllm_b200.qlora import Linear4bit
    g = torch.Generator(device=dev).manual_seed(seed)
    return Linear4bit.from_float(torch.randn(n, k, generator=g, device=dev) * 0.02, None)


def _same_for_every_fill(state, fn):
    ref = None
    for fill in FILLS:
        state["fill"] = fill
        out = [o.clone() for o in fn() if o is not None]
        _check_guards(state)
        if ref is None:
            ref = out
            continue
        for i, (o, e) in enumerate(zip(out, ref)):
            assert torch.equal(o, e), f"output {i} changed with workspace fill {fill:#x}"


@pytest.mark.parametrize("m", [1, 40, 300])
def test_swiglu_entries_workspace_contents_and_bounds(cuda_dev, guarded_workspace, m):
    from fitllm_b200 import ops
    from fitllm_b200.qlora import swiglu_forward
    n, k = 512, 256
    lg, lu, ld = _nf4(n, k, 1, cuda_dev), _nf4(n, k, 2, cuda_dev), _nf4(k, n, 3, cuda_dev)
    g = torch.Generator(device=cuda_dev).manual_seed(m)
    x = torch.randn(m, k, generator=g, device=cuda_dev).bfloat16()
    dy = torch.randn(m, k, generator=g, device=cuda_dev).bfloat16()
    if m <= 64:
        _same_for_every_fill(guarded_workspace, lambda: [swiglu_forward(lg, lu, x)])
    else:
        _same_for_every_fill(guarded_workspace,
                             lambda: list(ops.nf4_gateup_swiglu(x, lg.wref(), lu.wref(), keep_gate_up=True)))
        gate = torch.randn(m, n, generator=g, device=cuda_dev).bfloat16()
        up = torch.randn(m, n, generator=g, device=cuda_dev).bfloat16()
        _same_for_every_fill(guarded_workspace, lambda: list(ops.nf4_down_dswiglu(dy, ld.wref(), gate, up)))


def test_verify_attention_and_clip_workspace_contents_and_bounds(cuda_dev, guarded_workspace):
    from fitllm_b200 import ops
    g = torch.Generator(device=cuda_dev).manual_seed(5)
    b, t, h, kvh, d, prefix, cap = 2, 5, 8, 2, 128, 700, 768
    q = torch.randn(b, t, h, d, generator=g, device=cuda_dev).bfloat16()
    kc = torch.randn(b, kvh, cap, d, generator=g, device=cuda_dev).bfloat16()
    vc = torch.randn(b, kvh, cap, d, generator=g, device=cuda_dev).bfloat16()
    _same_for_every_fill(guarded_workspace, lambda: [ops.verify_attention(q, kc, vc, prefix)])
    flat = torch.randn(1 << 20, generator=g, device=cuda_dev)
    _same_for_every_fill(guarded_workspace, lambda: [ops.grad_clip_coef(flat, 1.0)])
