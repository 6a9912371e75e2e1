"""Sharded weight upload on two GPUs: each rank copies its 1/G byte range of a
layer arena from pinned host memory and one NCCL all-gather completes the
device slot; the slot must equal the layer's tensors byte for byte on every
rank, with each rank holding only its byte range in pinned host memory.
Runs two NCCL ranks as child processes (skipped with fewer than two GPUs)."""
import os
import subprocess
import sys
import textwrap

import pytest
import torch

pytestmark = pytest.mark.gpu

_CHILD = textwrap.dedent("""
    import datetime, os, sys, torch, torch.distributed as dist
    sys.path.insert(0, os.environ["FITQ_ROOT"])
    rank = int(os.environ["RANK"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    from fitllm_b200.scheduler import ShardScheduler
    g = torch.Generator().manual_seed(3)
    layers = [{"w": torch.randint(0, 256, (1_000_003,), generator=g, dtype=torch.uint8),
               "b": torch.randn(777, generator=g)} for _ in range(3)]
    sched = ShardScheduler(3, torch.device("cuda", rank), ring_slots=2)
    assert sched.shard_upload and sched.world == 2 and not sched.store_full
    for l, t in enumerate(layers):
        sched.add_layer(l, t)
    # each rank pins only its half of every arena
    assert sched.host_bytes() <= sum(sched.layer_bytes(l) for l in range(3)) // 2 + 3 * 256
    for l in range(3):
        dev = sched.get_layer_tensors(l)
        for k, v in layers[l].items():
            assert torch.equal(dev[k].cpu(), v), (rank, l, k)
        sched.release(l)
    torch.cuda.synchronize()
    dist.barrier(device_ids=[rank])
    dist.destroy_process_group()
    print("ok", rank)
""")


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sharded_upload_two_ranks(tmp_path):
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    script = tmp_path / "child.py"
    script.write_text(_CHILD)
    procs = []
    for rank in range(2):
        env = dict(os.environ, RANK=str(rank), WORLD_SIZE="2", LOCAL_RANK=str(rank),
                   MASTER_ADDR="127.0.0.1", MASTER_PORT="29533", FITQ_ROOT=root,
                   NCCL_NVLS_ENABLE="0")
        procs.append(subprocess.Popen([sys.executable, str(script)], env=env,
                                      stdout=subprocess.PIPE, stderr=subprocess.STDOUT))
    outs = [p.communicate(timeout=240)[0].decode() for p in procs]
    for rank, (p, o) in enumerate(zip(procs, outs)):
        assert p.returncode == 0, o[-2000:]
        assert f"ok {rank}" in o


_CHILD_STEP = textwrap.dedent("""
    import datetime, os, sys, torch, torch.distributed as dist
    sys.path.insert(0, os.environ["FITQ_ROOT"])
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    from fitllm_b200.distributed import LoRAGradComm, microbatch_range
    from fitllm_b200.engine import ShardStationaryEngine, build_synthetic_model
    from fitllm_b200.layer import LayerConfig
    from fitllm_b200.lm_head import random_lm_head
    from fitllm_b200.optimizer import ShardOptimizer
    cfg = LayerConfig(hidden=256, heads=4, kv_heads=2, head_dim=64, intermediate=512, lora_rank=16,
                      lora_alpha=32.0, lora_targets=("q_proj", "v_proj"), vocab=2048)
    sched, store = build_synthetic_model(cfg, 2, dev, seed=3)
    eng = ShardStationaryEngine(cfg, sched, store, dev, comm=LoRAGradComm(store))
    opt = ShardOptimizer(store)
    head = random_lm_head(cfg.hidden, cfg.vocab, dev, seed=4)
    g = torch.Generator(device=dev).manual_seed(5)
    ids = torch.randint(0, cfg.vocab, (4, 65), generator=g, device=dev)
    emb = (torch.randn(cfg.vocab, cfg.hidden, generator=g, device=dev) * 0.02).bfloat16()
    a, b = microbatch_range(4, rank, world)
    h0, labels = emb[ids[a:b, :64]].contiguous(), ids[a:b, 1:].contiguous()
    for _ in range(2):
        store.zero_grad()
        eng.step_with_loss(h0, labels, head, grad_accum=4)
        opt.step()
    torch.cuda.synchronize()
    flat = store.param.detach().clone()
    allp = [torch.empty_like(flat) for _ in range(world)]
    dist.all_gather(allp, flat)
    same = all(torch.equal(allp[0], p) for p in allp)
    torch.save(flat.cpu(), os.environ["FITQ_OUT"] + f".{world}.{rank}")
    dist.barrier(device_ids=[rank])
    dist.destroy_process_group()
    print("ok", rank, "identical" if same else "DIFFERENT")
""")


def _run_ranks(tmp_path, world, port, script_text):
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    script = tmp_path / f"child_{world}.py"
    script.write_text(script_text)
    procs = []
    for rank in range(world):
        env = dict(os.environ, RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                   MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), FITQ_ROOT=root,
                   NCCL_NVLS_ENABLE="0", FITQ_OUT=str(tmp_path / "params"))
        procs.append(subprocess.Popen([sys.executable, str(script)], env=env,
                                      stdout=subprocess.PIPE, stderr=subprocess.STDOUT))
    outs = [p.communicate(timeout=300)[0].decode() for p in procs]
    for rank, (p, o) in enumerate(zip(procs, outs)):
        assert p.returncode == 0, o[-3000:]
        assert f"ok {rank}" in o, o[-2000:]
    return outs


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_replicas_identical_after_steps(tmp_path):
    """Two data-parallel ranks (2 of 4 micro-batches each, per-layer NCCL
    all-reduce of the LoRA grads, identical clip + AdamW) end two steps with
    bit-identical adapters, and match a single-rank run of all 4 micro-batches
    within fp32 summation-order noise."""
    outs = _run_ranks(tmp_path, 2, 29541, _CHILD_STEP)
    assert all("identical" in o for o in outs)
    _run_ranks(tmp_path, 1, 29542, _CHILD_STEP)
    p2 = torch.load(tmp_path / "params.2.0")
    p1 = torch.load(tmp_path / "params.1.0")
    assert float((p2 - p1).norm() / p1.norm()) < 1e-4
