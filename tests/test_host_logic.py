"""Host-side logic on CPU (no GPU): the C-ABI library loads and exports every
symbol include/fitq.h declares, reference-API behaviour of LoRALinear /
LoRAManager on dense bases (restating fitllm's own tests), the golden outputs
of FitLLM's pure-torch code, QuantState serialisation, the shard store
layout, micro-batch splitting, and the per-layer gradient all-reduce on two
gloo ranks."""
import ctypes
import json
import os
import re
import socket
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.nn as nn

ROOT = Path(__file__).resolve().parent.parent
GOLD = ROOT / "tests" / "golden"


# ---------------------------------------------------------------- C ABI
def test_library_loads_and_exports_header_symbols():
    from fitllm_b200 import _lib, build
    build.build()
    header = (ROOT / "include" / "fitq.h").read_text()
    declared = set(re.findall(r"FITQ_API\s+[\w\s\*]+?\b(fitq_\w+)\s*\(", header))
    assert len(declared) >= 16
    L = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in declared:
        assert hasattr(L, name), name
    assert set(_lib.SIGNATURES) == declared
    assert _lib.version().startswith("fitq")


def test_attention_abi_checks_arguments_before_the_device():
    """The training attention's shape, head_dim and alignment checks run on
    the host before any CUDA call (pointers are never dereferenced there), so
    they answer without a GPU.  Every call here is refused before launch, so
    the stand-in pointers are safe on a machine with a GPU too."""
    from fitllm_b200 import _lib
    L = _lib.load()
    p = 1 << 20  # a 16-byte-aligned stand-in address, never touched
    assert L.fitq_attention_fwd(None, p, p, p, p, 1, 128, 4, 2, 128, None) == 1      # NULL
    assert L.fitq_attention_fwd(p, p, p, p, p, 1, 100, 4, 2, 128, None) == 2         # S % 64
    assert L.fitq_attention_fwd(p, p, p, p, p, 1, 128, 6, 4, 128, None) == 2         # H % KVH
    assert L.fitq_attention_fwd(p, p, p, p, p, 0, 128, 4, 2, 128, None) == 2         # batch
    assert L.fitq_attention_fwd(p, p, p, p, p, 1, 128, 4, 2, 96, None) == 4          # head_dim
    assert L.fitq_attention_fwd(p + 8, p, p, p, p, 1, 128, 4, 2, 128, None) == 3     # alignment
    assert b"16-byte" in L.fitq_last_error()
    ws = L.fitq_attention_bwd_workspace(2, 256, 40)
    assert ws == 2 * 256 * 40 * 4 and L.fitq_attention_bwd_workspace(0, 256, 40) == 0
    assert L.fitq_attention_bwd(p, p, p, p, p, p, p, p, p, 2, 256, 40, 8, 128, p, ws - 1, None) == 5
    assert b"workspace" in L.fitq_last_error()


def test_abi_rejects_bad_arguments_without_a_device():
    from fitllm_b200 import _lib
    L = _lib.load()
    w = _lib.Nf4WeightC(packed=None, quant_map=None, n_out=64, k_in=64)
    rc = L.fitq_nf4_dequant(ctypes.byref(w), None, 0, 0, None)
    assert rc == 1  # FITQ_ERR_ARG: checked before any device call
    w2 = _lib.Nf4WeightC(packed=16, quant_map=16, absmax_f32=16, n_out=64, k_in=100)
    assert L.fitq_nf4_dequant(ctypes.byref(w2), 16, 0, 0, None) == 2  # K % 64 != 0
    assert L.fitq_gemm_bf16_tn(16, 16, 16, None, 128, 100, 64, None) == 2  # N % 16 != 0
    assert b"N % 16 == 0" in L.fitq_last_error()
    import os
    try:
        # NF4 decoded inside the GEMM: no dequantised copy of W in the workspace
        os.environ["FITQ_NF4_FUSED"] = "1"
        assert L.fitq_qlora_fwd_workspace(512, 5120, 5120, 16) < 5120 * 5120 // 2
        assert L.fitq_qlora_bwd_workspace(512, 5120, 5120, 16) < 5120 * 5120 // 2
        # the dequant + bf16 GEMM path holds W (bf16) in the workspace
        os.environ["FITQ_NF4_FUSED"] = "0"
        assert L.fitq_qlora_fwd_workspace(512, 5120, 5120, 16) > 5120 * 5120 * 2
        assert L.fitq_qlora_bwd_workspace(512, 5120, 5120, 16) > 5120 * 5120 * 2
    finally:
        os.environ.pop("FITQ_NF4_FUSED", None)
    # shapes the fused GEMM does not take (N % 128 != 0) keep the dequant path
    assert L.fitq_qlora_fwd_workspace(512, 320, 256, 16) > 320 * 256 * 2
    # by default the fused GEMM takes few-row GEMMs whose output side is 4x the
    # reduction (gate/up forward, down_proj dX at M <= 2048), dequant otherwise
    assert L.fitq_qlora_fwd_workspace(2048, 27648, 5120, 0) < 27648 * 5120 // 2
    assert L.fitq_qlora_bwd_workspace(2048, 5120, 27648, 0) < 27648 * 5120 // 2
    assert L.fitq_qlora_fwd_workspace(4096, 27648, 5120, 0) >= 27648 * 5120 * 2
    assert L.fitq_qlora_fwd_workspace(2048, 5120, 27648, 0) >= 27648 * 5120 * 2
    assert L.fitq_qlora_bwd_workspace(2048, 27648, 5120, 0) >= 27648 * 5120 * 2


# ---------------------------------------------------------------- reference API
class _Tiny(nn.Module):
    def __init__(self, h=16):
        super().__init__()
        self.q_proj = nn.Linear(h, h, bias=False)
        self.k_proj = nn.Linear(h, h, bias=False)
        self.v_proj = nn.Linear(h, h, bias=False)
        self.o_proj = nn.Linear(h, h, bias=False)
        self.mlp = nn.Linear(h, h, bias=False)

    def forward(self, x):
        return self.o_proj(self.q_proj(x) + self.k_proj(x) + self.v_proj(x)) + self.mlp(x)


def test_lora_linear_reference_behaviour():
    from fitllm_b200.lora import LoRALinear
    base = nn.Linear(16, 32, bias=False)
    lora = LoRALinear(base, rank=4, alpha=8.0)
    assert lora(torch.randn(2, 8, 16)).shape == (2, 8, 32)
    assert lora.scale == 2.0
    assert torch.all(lora.lora_B == 0) and lora.lora_A.abs().sum() > 0
    assert not base.weight.requires_grad and lora.lora_A.requires_grad


def test_lora_manager_inject_state_dict_and_grads():
    from fitllm_b200.lora import LoRALinear, LoRAManager
    torch.manual_seed(0)
    model = _Tiny()
    mgr = LoRAManager()
    mgr.inject_lora(model, rank=2, alpha=4.0, targets=("q_proj", "v_proj"))
    assert isinstance(model.q_proj, LoRALinear) and isinstance(model.k_proj, nn.Linear)
    assert mgr.num_lora_layers == 2
    mgr.freeze_base_model(model)
    out = model(torch.randn(3, 16)).sum()
    out.backward()
    named = dict(model.named_parameters())
    for n, p in named.items():
        if "lora_" in n:
            assert p.grad is not None
        else:
            assert p.grad is None
    sd = mgr.state_dict()
    assert set(sd) == {"q_proj.lora_A", "q_proj.lora_B", "v_proj.lora_A", "v_proj.lora_B"}
    model2 = _Tiny()
    mgr2 = LoRAManager()
    mgr2.inject_lora(model2, rank=2, alpha=4.0, targets=("q_proj", "v_proj"))
    mgr2.load_state_dict(sd)
    for k, v in mgr2.state_dict().items():
        assert torch.equal(v, sd[k])
    assert len(list(mgr.trainable_parameters())) == 4


def test_lora_linear_matches_reference_golden():
    """Dense-base LoRALinear against fitllm.lora.LoRALinear outputs."""
    from fitllm_b200.lora import LoRALinear
    d = torch.load(GOLD / "reference_torch.pt", weights_only=False)["lora"]
    base = nn.Linear(32, 48, bias=False)
    lora = LoRALinear(base, rank=16, alpha=32.0)
    with torch.no_grad():
        base.weight.copy_(d["base_w"])
        lora.lora_A.copy_(d["A"])
        lora.lora_B.copy_(d["B"])
    x = d["x"].clone().requires_grad_(True)
    y = lora(x)
    y.backward(d["gy"])
    assert torch.equal(y, d["y"])
    assert torch.equal(x.grad, d["gx"])
    assert torch.equal(lora.lora_A.grad, d["gA"]) and torch.equal(lora.lora_B.grad, d["gB"])


def test_cosine_lr_matches_reference_golden():
    from fitllm_b200.optimizer import cosine_lr_scale
    for s, w, m, v in torch.load(GOLD / "reference_torch.pt", weights_only=False)["cosine"]:
        assert cosine_lr_scale(s, w, m) == v


def _adamw_restated(p, g, m, v, t, lr, b1, b2, eps, wd):
    m = b1 * m + (1 - b1) * g
    v = b2 * v + (1 - b2) * g * g
    mh, vh = m / (1 - b1 ** t), v / (1 - b2 ** t)
    return p - lr * (mh / (vh.sqrt() + eps) + wd * p), m, v


def test_adamw_order_matches_reference_golden():
    """The update order the device kernel implements (restated in fp32 torch)
    reproduces ShardOptimizer.step_from_memory bit for bit."""
    d = torch.load(GOLD / "reference_torch.pt", weights_only=False)["adamw"]
    layer_of = {n: int(n.split("layers.")[1].split(".")[0]) for n in d["names"]}
    for n in d["names"]:
        p, m, v = d["init"][n].clone(), torch.zeros(4, 6), torch.zeros(4, 6)
        for t, grads in enumerate(d["grads"], start=1):
            local = n.split(f"layers.{layer_of[n]}.")[1]
            p, m, v = _adamw_restated(p, grads[layer_of[n]][local], m, v, t, d["lr"], d["beta1"],
                                      d["beta2"], d["eps"], d["wd"])
        assert torch.equal(p, d["final"][n]), n


def test_clip_golden():
    d = torch.load(GOLD / "reference_torch.pt", weights_only=False)["clip"]
    flat = torch.cat([d["before"][0]["a"], d["before"][1]["b"]]).double()
    norm = float(flat.norm())
    assert abs(norm - d["norm"]) / d["norm"] < 1e-6
    coef = d["max_norm"] / (norm + 1e-6)
    assert torch.allclose(d["before"][1]["b"] * coef, d["after"][1]["b"], rtol=1e-6)


# ---------------------------------------------------------------- formats
def test_quant_state_dict_round_trip():
    from fitllm_b200.nf4 import QuantState
    qs = QuantState(absmax=torch.arange(16, dtype=torch.uint8), shape=(8, 128),
                    quant_map=torch.linspace(-1, 1, 16), nested_absmax=torch.tensor([0.5]),
                    nested_quant_map=torch.linspace(-1, 1, 256), offset=0.125)
    d = qs.as_dict(packed=True)
    assert set(d) == {"absmax", "quant_map", "nested_absmax", "nested_quant_map",
                      "quant_state.bitsandbytes__nf4"}
    meta = json.loads(bytes(d["quant_state.bitsandbytes__nf4"].tolist()))
    assert meta["quant_type"] == "nf4" and meta["blocksize"] == 64 and meta["nested_offset"] == 0.125
    back = QuantState.from_dict(d, device="cpu")
    assert back.shape == (8, 128) and back.offset == 0.125 and back.nested
    assert torch.equal(back.absmax, qs.absmax)


def test_shard_store_layout_drops_lora_keys():
    from fitllm_b200.scheduler import ShardScheduler
    s = ShardScheduler(2, "cpu", ring_slots=2, pin_memory=False)
    meta = torch.tensor(list(json.dumps({"shape": [4, 64], "nested_offset": 0.5}).encode()),
                        dtype=torch.uint8)
    t = {"a.weight": torch.arange(128, dtype=torch.uint8).view(-1, 1),
         "a.weight.absmax": torch.ones(4, dtype=torch.uint8),
         "a.weight.quant_state.bitsandbytes__nf4": meta,
         "n.weight": torch.randn(64).bfloat16(),
         "q.lora_A.default.weight": torch.randn(2, 2)}
    nb = s.add_layer(0, t)
    assert nb % 256 == 0
    host = s.host_tensors(0)
    assert "q.lora_A.default.weight" not in host
    assert torch.equal(host["a.weight"], t["a.weight"]) and torch.equal(host["n.weight"], t["n.weight"])
    assert s.quant_meta(0)["a.weight"]["nested_offset"] == 0.5


def test_ring_slot_map_advances_on_invalidate():
    from fitllm_b200.scheduler import ShardScheduler
    s = ShardScheduler(3, "cpu", ring_slots=2, pin_memory=False)
    assert [s.slot_of(l) for l in range(3)] == [0, 1, 0]
    s.invalidate()
    assert [s.slot_of(l) for l in range(3)] == [1, 0, 1]
    s.invalidate()
    assert [s.slot_of(l) for l in range(3)] == [0, 1, 0]


def test_microbatch_split():
    from fitllm_b200.distributed import microbatch_range
    for n in (16, 15, 3):
        for world in (1, 2, 4, 8):
            spans = [microbatch_range(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1


# ---------------------------------------------------------------- multi-rank (gloo)
def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, q):
    import torch.distributed as dist
    from fitllm_b200.distributed import LoRAGradComm, microbatch_range
    from fitllm_b200.optimizer import LoRAStore
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    store = LoRAStore(3, [("a", (4, 8)), ("b", (8, 4))], "cpu")
    # per-rank grads: each rank owns micro-batches [s, e); grad of mb i is i+1 everywhere
    s, e = microbatch_range(6, rank, world)
    for layer in range(3):
        store.layer_slice(store.grad, layer).fill_(float(sum(range(s + 1, e + 1))) * (layer + 1))
    comm = LoRAGradComm(store)
    for layer in reversed(range(3)):
        comm.allreduce_layer(layer)
    comm.wait()
    uniform = all(bool(torch.all(store.layer_slice(store.grad, l) == store.layer_slice(store.grad, l)[0]))
                  for l in range(3))
    q.put((rank, [float(store.layer_slice(store.grad, l)[0]) for l in range(3)], uniform))
    dist.destroy_process_group()


def test_per_layer_allreduce_two_gloo_ranks():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    total = sum(range(1, 7))
    for _, vals, uniform in res:
        assert vals == [total * 1.0, total * 2.0, total * 3.0]
        assert uniform


def _rank_store_main(rank, world, port, q):
    import torch.distributed as dist
    from fitllm_b200.scheduler import ShardScheduler, shard_ranges
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    g = torch.Generator().manual_seed(5)
    layers = [{"w": torch.randint(0, 256, (10_001 + 97 * l,), generator=g, dtype=torch.uint8),
               "b": torch.randn(33, generator=g).bfloat16()} for l in range(3)]
    part = ShardScheduler(3, "cpu", pin_memory=False)
    full = ShardScheduler(3, "cpu", pin_memory=False, store_full=True)
    ok = part.shard_upload and not part.store_full and full.store_full
    for l, t in enumerate(layers):
        part.add_layer(l, t)
        full.add_layer(l, t)
        _, ranges = shard_ranges(full.layer_bytes(l), world)
        a, b = ranges[rank]
        ok = ok and part.layer_bytes(l) == full.layer_bytes(l)
        ok = ok and torch.equal(part._host[l], full._host[l][a:b])
        ok = ok and part.upload_bytes(l) == b - a
    q.put((rank, ok, part.host_bytes(), full.host_bytes()))
    dist.destroy_process_group()


def test_sharded_host_store_keeps_only_the_rank_range():
    """With data-parallel ranks each rank pins only the byte range of every
    layer arena that it uploads (its part of the in-place all-gather); the
    range equals the same bytes of the whole arena."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_store_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok for _, ok, _, _ in res)
    assert sum(h for _, _, h, _ in res) == res[0][3]  # the two ranges make up the arenas


def test_shard_ranges_cover_arena():
    """The per-rank upload ranges tile the arena exactly, in equal 256-byte
    aligned chunks (short or empty at the end)."""
    from fitllm_b200.scheduler import shard_ranges
    for total in (1, 255, 256, 257, 251_531_520, 4096 * 7 + 13):
        for world in (1, 2, 3, 4, 8):
            chunk, ranges = shard_ranges(total, world)
            assert chunk % 256 == 0 and chunk * world >= total
            pos = 0
            for i, (a, b) in enumerate(ranges):
                assert a == min(i * chunk, total) and a == pos and a <= b <= total
                pos = b
            assert pos == total


def _rank_fail_main(rank, world, port, q, mode):
    """Rank 1 fails (mode "raise": raises after joining, before the first
    layer's all-reduce; "absent": never joins the group); rank 0 must end
    with an error from the process group's short timeout instead of hanging."""
    import time
    from fitllm_b200.distributed import LoRAGradComm, init_from_env
    from fitllm_b200.optimizer import LoRAStore
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    if rank == 1 and mode == "absent":
        q.put((rank, "absent", 0.0))
        return
    t0 = time.time()
    try:
        init_from_env(backend="gloo", timeout_s=5.0)
        if rank == 1:
            raise RuntimeError("injected failure on rank 1")
        store = LoRAStore(2, [("a", (4, 8))], "cpu")
        comm = LoRAGradComm(store)
        for layer in reversed(range(2)):
            comm.allreduce_layer(layer)
        comm.wait()
        q.put((rank, "ok", time.time() - t0))
    except Exception as e:  # the failure the test expects on rank 0
        q.put((rank, type(e).__name__, time.time() - t0))
        if rank == 1:
            q.close()
            q.join_thread()  # the report is sent before the abrupt exit
            os._exit(3)  # leave without tearing the group down, like a crashed rank


@pytest.mark.parametrize("mode", ["raise", "absent"])
def test_failed_rank_ends_collectives_with_an_error(mode):
    """Failure detection on the host: when one rank raises or never joins,
    the surviving rank's group initialisation or per-layer all-reduce ends
    with an exception within the process-group timeout (5 s here), so a
    training job fails fast instead of hanging."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_fail_main, args=(r, 2, port, q, mode)) for r in range(2)]
    for p in procs:
        p.start()
    res = {r: (status, t) for r, status, t in (q.get(timeout=120) for _ in procs)}
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[0][0] != "ok", res
    assert res[0][1] < 60.0, res
    if mode == "raise":
        assert res[1][0] == "RuntimeError"


def test_attention_wrapper_rejects_bad_tensors_before_the_library():
    """The training attention's Python wrappers check dtype, layout and shapes
    themselves (the C ABI only sees pointers); every case raises before any
    device work, so this runs without a GPU."""
    import pytest
    import torch
    from fitllm_b200.layer_ops import attention_backward, attention_forward
    q = torch.zeros(1, 64, 4, 128, dtype=torch.bfloat16)
    k = torch.zeros(1, 64, 2, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        attention_forward(q, k, k)                      # CPU tensors
    with pytest.raises(ValueError, match="match"):
        attention_forward(q, k[:, :32], k)              # S mismatch
    with pytest.raises(ValueError, match="head_dim"):
        attention_forward(q[0], k, k)                   # not 4-D
    with pytest.raises(ValueError, match="CUDA"):
        attention_backward(q.float(), k, k, q, torch.zeros(1, 4, 64), q)
