"""Sharded weight upload on two GPUs: each rank copies its 1/G byte range of a
layer arena from pinned host memory and one NCCL all-gather completes the
device slot; the slot must equal the host arena byte for byte on every rank.
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
    assert sched.shard_upload and sched.world == 2
    for l, t in enumerate(layers):
        sched.add_layer(l, t)
    for l in range(3):
        dev = sched.get_layer_tensors(l)
        host = sched.host_tensors(l)
        for k in host:
            assert torch.equal(dev[k].cpu(), host[k]), (rank, l, k)
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
