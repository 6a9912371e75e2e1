"""The SwiGLU MLP with the activation fused into the tcgen05 GEMMs.

fitq_nf4_gateup_swiglu (gate and up as one GEMM, SwiGLU in the epilogue) and
fitq_nf4_down_dswiglu (down_proj's dX GEMM with the SwiGLU backward in the
epilogue) are bit-identical to the separate calls they replace: two
fitq_qlora_fwd + fitq_swiglu_fwd, and fitq_qlora_bwd's dX + fitq_swiglu_bwd.
The fused MLP module's forward is bit-identical to the unfused module's; its
dx sums the gate and up dX in fp32 (one rounding instead of two), so it is
checked against the unfused dx to a few bf16 ulps and against an fp32
restatement at the 1e-2 relative contract.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

REL_TOL = 1e-2


def _weight(n, k, seed, dev):
    from fitllm_b200.qlora import Linear4bit
    g = torch.Generator(device=dev).manual_seed(seed)
    return Linear4bit.from_float(torch.randn(n, k, generator=g, device=dev) * 0.02, None).wref()


SHAPES = [(256, 1024, 512), (300, 384, 256), (130, 256, 1024), (512, 27648, 5120)]


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_gateup_swiglu_bit_identical(cuda_dev, m, n, k):
    from fitllm_b200 import ops
    from fitllm_b200.layer_ops import swiglu
    wg = _weight(n, k, 31 + n, cuda_dev)
    wu = _weight(n, k, 57 + n, cuda_dev)
    g = torch.Generator(device=cuda_dev).manual_seed(m)
    x = torch.randn(m, k, generator=g, device=cuda_dev).bfloat16()
    act, gate, up = ops.nf4_gateup_swiglu(x, wg, wu, keep_gate_up=True)
    act_only, none_g, none_u = ops.nf4_gateup_swiglu(x, wg, wu, keep_gate_up=False)
    gate2, _ = ops.qlora_forward(x, wg, None, None, 1.0)
    up2, _ = ops.qlora_forward(x, wu, None, None, 1.0)
    act2 = swiglu(gate2, up2)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    assert none_g is None and none_u is None
    assert torch.equal(gate, gate2)
    assert torch.equal(up, up2)
    assert torch.equal(act, act2)
    assert torch.equal(act_only, act2)


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_down_dswiglu_bit_identical(cuda_dev, m, n, k):
    """down_proj: [k_hidden, n_intermediate] as (n_out = k, k_in = n)."""
    from fitllm_b200 import ops
    from fitllm_b200.layer_ops import SwiGLUFn
    wd = _weight(k, n, 91 + n, cuda_dev)
    g = torch.Generator(device=cuda_dev).manual_seed(m + 1)
    dy = torch.randn(m, k, generator=g, device=cuda_dev).bfloat16()
    gate = (torch.randn(m, n, generator=g, device=cuda_dev) * 2).bfloat16()
    up = torch.randn(m, n, generator=g, device=cuda_dev).bfloat16()
    d_gate, d_up = ops.nf4_down_dswiglu(dy, wd, gate, up)
    d_act, _, _ = ops.qlora_backward(None, dy, wd, None, None, 1.0)
    gate_r = gate.clone().requires_grad_(True)
    up_r = up.clone().requires_grad_(True)
    SwiGLUFn.apply(gate_r, up_r).backward(d_act)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    assert torch.equal(d_gate, gate_r.grad)
    assert torch.equal(d_up, up_r.grad)


@pytest.mark.parametrize("m,hidden,inter", [(2, 512, 1024), (1, 640, 384)])
def test_mlp_module_fused_vs_unfused(cuda_dev, m, hidden, inter):
    from fitllm_b200.layer import MLP, LayerConfig
    from fitllm_b200.qlora import Linear4bit
    cfg = LayerConfig(hidden=hidden, intermediate=inter, heads=4, kv_heads=2, head_dim=hidden // 4)
    mlp = MLP(cfg, device=cuda_dev)
    assert not mlp.fused  # opt-in (FITQ_MLP_FUSED=1)
    g = torch.Generator(device=cuda_dev).manual_seed(inter)
    dense = {}
    for name, (o, i) in {"gate_proj": (inter, hidden), "up_proj": (inter, hidden),
                         "down_proj": (hidden, inter)}.items():
        w = torch.randn(o, i, generator=g, device=cuda_dev) * 0.03
        lin = Linear4bit.from_float(w, None)
        setattr(mlp, name, lin)
        dense[name] = lin.dequantize(torch.bfloat16).float()
    seq = 96
    x = (torch.randn(m, seq, hidden, generator=g, device=cuda_dev)).bfloat16()
    res = (torch.randn(m, seq, hidden, generator=g, device=cuda_dev)).bfloat16()
    dy = (torch.randn(m, seq, hidden, generator=g, device=cuda_dev)).bfloat16()

    def run(fused, fused_backward=True):
        mlp.fused = fused
        mlp.fused_backward = fused_backward
        xi = x.clone().requires_grad_(True)
        ri = res.clone().requires_grad_(True)
        out = mlp(xi, ri)
        out.backward(dy)
        return out.detach(), xi.grad, ri.grad

    yf, dxf, drf = run(True)
    yh, dxh, drh = run(True, fused_backward=False)
    yu, dxu, dru = run(False)
    torch.cuda.synchronize()
    # forward fused, backward through the separate SwiGLU kernel: same bits as fused
    assert torch.equal(yh, yf) and torch.equal(dxh, dxf) and torch.equal(drh, drf)
    assert torch.equal(yf, yu)
    assert torch.equal(drf, dru)
    # the two dx sums differ by the rounding of one bf16 term: a few bf16 ulps
    assert float((dxf.float() - dxu.float()).norm() / dxu.float().norm()) < 4e-3
    # fp32 restatement
    xr = x.float().reshape(-1, hidden).requires_grad_(True)
    gr = xr @ dense["gate_proj"].T
    ur = xr @ dense["up_proj"].T
    yr = (torch.nn.functional.silu(gr) * ur) @ dense["down_proj"].T + res.float().reshape(-1, hidden)
    yr.backward(dy.float().reshape(-1, hidden))
    rel = lambda a, b: float((a.float().reshape(b.shape) - b).norm() / b.norm())
    assert rel(yf, yr.detach()) < REL_TOL
    assert rel(dxf, xr.grad) < REL_TOL
