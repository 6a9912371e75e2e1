"""Shard files (fitllm_b200/shards.py): the reference's safetensors + .sha256
layout (fitllm/scheduler.py:21-67, fitllm/model.py:25-83), checksum errors,
group files and the one-time load into the pinned host store."""
import hashlib
import json

import pytest
import torch

from fitllm_b200 import shards
from fitllm_b200.scheduler import ShardScheduler


def _layer_dict(seed: int):
    g = torch.Generator().manual_seed(seed)
    meta = json.dumps({"quant_type": "nf4", "blocksize": 64, "shape": [64, 128],
                       "nested_offset": 0.01}).encode()
    return {
        "self_attn.q_proj.weight": torch.randint(0, 256, (64 * 128 // 2, 1), generator=g, dtype=torch.uint8),
        "self_attn.q_proj.weight.absmax": torch.randint(0, 256, (128,), generator=g, dtype=torch.uint8),
        "self_attn.q_proj.weight.quant_map": torch.randn(16, generator=g),
        "self_attn.q_proj.weight.quant_state.bitsandbytes__nf4": torch.tensor(list(meta), dtype=torch.uint8),
        "self_attn.q_proj.bias": torch.randn(64, generator=g).bfloat16(),
        "self_attn.q_proj.lora_A.default.weight": torch.randn(4, 128, generator=g),
        "input_layernorm.weight": torch.ones(128, dtype=torch.bfloat16),
    }


def test_save_load_roundtrip_and_sidecar(tmp_path):
    d = _layer_dict(1)
    p = tmp_path / shards.shard_file_name(0)
    shards.save_shard_with_checksum(d, p)
    assert p.name == "layer_000_weights.safetensors"
    side = p.with_suffix(".sha256")
    assert side.read_text() == hashlib.sha256(p.read_bytes()).hexdigest()
    back = shards.load_shard_with_checksum(p)
    assert set(back) == set(d)
    for k in d:
        assert back[k].dtype == d[k].dtype and torch.equal(back[k], d[k])


def test_checksum_mismatch_raises(tmp_path):
    p = tmp_path / shards.shard_file_name(3)
    shards.save_shard_with_checksum(_layer_dict(2), p)
    raw = bytearray(p.read_bytes())
    raw[-1] ^= 0xFF  # flip the last data byte
    p.write_bytes(bytes(raw))
    with pytest.raises(RuntimeError, match="Checksum mismatch"):
        shards.load_shard_with_checksum(p)
    shards.load_shard_with_checksum(p, verify=False)  # no check requested
    p.with_suffix(".sha256").unlink()
    shards.load_shard_with_checksum(p)  # no sidecar: nothing to compare, as in the reference


def test_group_files_names_and_keys(tmp_path):
    layers = [_layer_dict(10 + i) for i in range(5)]
    assert shards.write_layer_shards(layers, tmp_path, group_size=2) == 5
    names = sorted(x.name for x in tmp_path.glob("*.safetensors"))
    assert names == ["layer_000-001_weights.safetensors", "layer_002-003_weights.safetensors",
                     "layer_004-004_weights.safetensors"]
    t = shards.load_shard_with_checksum(tmp_path / names[1])
    assert "0.self_attn.q_proj.weight" in t and "1.input_layernorm.weight" in t
    per = shards.split_group(t, 2)
    assert torch.equal(per[1]["self_attn.q_proj.weight"], layers[3]["self_attn.q_proj.weight"])


@pytest.mark.parametrize("group_size", [1, 3])
def test_load_into_host_store(tmp_path, group_size):
    layers = [_layer_dict(20 + i) for i in range(4)]
    shards.write_layer_shards(layers, tmp_path, group_size=group_size)
    sched = ShardScheduler(4, "cpu", pin_memory=False)
    total = shards.load_shards_into(sched, tmp_path, 4, group_size=group_size, threads=2)
    assert total == sum(sched.layer_bytes(i) for i in range(4))
    for i in range(4):
        host = sched.host_tensors(i)
        assert not any("lora_" in k for k in host)  # adapters dropped (fitllm/forward.py:733-734)
        for k, v in layers[i].items():
            if "lora_" in k:
                continue
            assert torch.equal(host[k].view(v.dtype).view(v.shape), v), k
        assert sched.quant_meta(i)["self_attn.q_proj.weight"]["blocksize"] == 64


def test_missing_or_corrupt_shard_fails_before_loading(tmp_path):
    layers = [_layer_dict(30 + i) for i in range(3)]
    shards.write_layer_shards(layers, tmp_path)
    sched = ShardScheduler(3, "cpu", pin_memory=False)
    with pytest.raises(FileNotFoundError):
        shards.load_shards_into(sched, tmp_path, 4)
    p = tmp_path / shards.shard_file_name(1)
    raw = bytearray(p.read_bytes())
    raw[-2] ^= 1
    p.write_bytes(bytes(raw))
    with pytest.raises(RuntimeError, match="Checksum mismatch"):
        shards.load_shards_into(sched, tmp_path, 3)
    assert sched.num_layers == 3 and not sched._host  # nothing stored


def test_writer_copies_each_layer_before_the_next(tmp_path):
    """A producer that reuses one buffer for every layer (as the synthetic
    model generator does) still gets one file per layer with its own values."""
    buf = torch.zeros(8)

    def layers():
        for i in range(3):
            buf.fill_(float(i))
            yield {"w": buf}

    assert shards.write_layer_shards(layers(), tmp_path) == 3
    for i in range(3):
        t = shards.load_shard_with_checksum(tmp_path / shards.shard_file_name(i))
        assert torch.equal(t["w"], torch.full((8,), float(i)))
