"""Shard-stationary forward / backward over layers (FitLLM's training loop core).

Follows ForwardEngine.shard_stationary_forward (fitllm/forward.py:408-541) and
BackwardEngine.shard_stationary_backward (fitllm/backward.py:149-251):

* forward: for each layer, load its shard ONCE and run every micro-batch
  through it without autograd, keeping the boundary activation h_l;
* backward, layers in reverse: reload the shard, recompute the layer forward
  with autograd from h_l, back-propagate the upstream gradient, hand the
  gradient w.r.t. h_l to the next layer down, and accumulate the LoRA
  gradients of all micro-batches into that layer's gradient slice
  (_accumulate_grads_to_ram, fitllm/backward.py:287-299).

B200 differences (same mathematics):
* the micro-batches of a rank are stacked along the batch dimension, so each
  projection is ONE GEMM over all of them (optionally in chunks);
* shards stream through the scheduler's pinned-host -> device ring, with the
  next layer's upload overlapping the current layer's compute;
* activations and gradients stay in HBM (180 GB) instead of round-tripping
  through host memory per micro-batch;
* LoRA gradients accumulate in place in a flat fp32 device buffer, and each
  layer's slice is all-reduced across ranks as soon as its backward is queued;
* the recompute uses the same dtype and attention mask as the forward
  (the reference's recompute drops autocast and the mask,
  fitllm/backward.py:222-231, which its own notes call a bug);
* HBM budget instead of a fixed recompute: the forward runs WITH autograd for
  the last layers whose saved activations fit the budget
  (``keep_activations``), and the backward of those layers skips the
  recompute (identical values, one layer-forward of work less).  The other
  layers are recomputed as in the reference.  A kept graph references its
  layer's ring slot and LoRA slices; the backward re-loads the layer (same
  slot, same views) before using it.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Sequence

import torch

from .distributed import LoRAGradComm
from .layer import DecoderLayer, LayerConfig, add_lora_, rotary_tables
from .nf4 import QuantState
from .optimizer import LoRAStore
from .qlora import Linear4bit, Params4bit, QLoRALinear4bit
from .scheduler import ShardScheduler


def layer_shard(layer: DecoderLayer) -> Dict[str, torch.Tensor]:
    """The flat shard key set of one layer (fitllm/forward.py:95-109 layout),
    adapter keys excluded."""
    sd = {}
    for k, v in layer.state_dict().items():
        if "lora_A" in k or "lora_B" in k:
            continue
        sd[k.replace(".base_layer.", ".")] = v
    return sd


def bind_layer(layer: DecoderLayer, tensors: Dict[str, torch.Tensor], meta: Dict[str, dict]) -> None:
    """Point the template layer's weights at one shard's device tensors (no copies).

    The device-side counterpart of _reconstruct_layer_module +
    _restore_bnb_quant_state (fitllm/forward.py:723-762, :76-109)."""
    for name, mod in layer.projections():
        base: Linear4bit = mod.base_layer if isinstance(mod, QLoRALinear4bit) else mod
        key = name + ".weight"
        m = meta[key]
        qs = QuantState(
            absmax=tensors[key + ".absmax"], shape=(int(m["shape"][0]), int(m["shape"][1])),
            quant_map=tensors[key + ".quant_map"],
            nested_absmax=tensors.get(key + ".nested_absmax"),
            nested_quant_map=tensors.get(key + ".nested_quant_map"),
            offset=float(m.get("nested_offset", 0.0)))
        base.weight = Params4bit(tensors[key], qs)
        base._wref = None
        if base.bias is not None:
            base.bias.data = tensors[name + ".bias"]
    layer.input_layernorm.weight.data = tensors["input_layernorm.weight"]
    layer.post_attention_layernorm.weight.data = tensors["post_attention_layernorm.weight"]


def lora_entries(layer: DecoderLayer):
    return [(n, tuple(p.shape)) for n, p in layer.named_parameters() if "lora_" in n]


class ShardStationaryEngine:
    def __init__(self, cfg: LayerConfig, scheduler: ShardScheduler, store: LoRAStore, device,
                 comm: Optional[LoRAGradComm] = None, mb_chunk: Optional[int] = None,
                 keep_activations="auto", keep_budget_fraction: float = 0.75):
        """keep_activations: "auto" (as many trailing layers as fit in
        keep_budget_fraction of the free HBM), an int (that many trailing
        layers) or 0 (recompute every layer, the reference behaviour).
        The estimate per layer (saved_bytes_per_token) is ~8% below what
        autograd keeps; at 0.78 the 64-layer, 16 x 1024-token step kept 56
        layers and peaked at 163 GB of a 191.5 GB B200, so 0.75 leaves room
        for the backward's temporaries."""
        self.keep_activations = keep_activations
        self.keep_budget_fraction = keep_budget_fraction
        self._keep_cache = {}  # tokens -> layers kept ("auto")
        self._graphs: Dict[int, tuple] = {}
        self.last_kept = 0
        self.cfg = cfg
        self.scheduler = scheduler
        self.store = store
        self.device = torch.device(device)
        self.comm = comm
        self.mb_chunk = mb_chunk
        self.layer = DecoderLayer(cfg, device=self.device)
        add_lora_(self.layer, cfg.lora_rank, cfg.lora_alpha, cfg.lora_targets, seed=0)
        self.layer.eval()
        self._pe = None

    @property
    def num_layers(self) -> int:
        return self.scheduler.num_layers

    def position_embeddings(self, seq_len: int, dtype=torch.bfloat16):
        if self._pe is None or self._pe[0].shape[0] != seq_len:
            self._pe = rotary_tables(seq_len, self.cfg.head_dim, self.cfg.rope_theta, self.device)
        return self._pe

    def _load(self, l: int) -> None:
        t = self.scheduler.get_layer_tensors(l)
        bind_layer(self.layer, t, self.scheduler.quant_meta(l))
        self.store.bind(l, self.layer)

    def _chunks(self, b: int):
        c = self.mb_chunk or b
        return [(i, min(b, i + c)) for i in range(0, b, c)]

    def saved_bytes_per_token(self) -> int:
        """Autograd state one token leaves in a layer (bf16): normed input, T,
        q, k, v, attention output (+ LSE), post-attention residual, gate, up."""
        c = self.cfg
        qd, kvd = c.heads * c.head_dim, c.kv_heads * c.head_dim
        return 2 * (c.hidden + 2 * c.lora_rank + 2 * qd + 2 * kvd + c.hidden + 2 * c.intermediate) + 4 * c.heads

    def _layers_to_keep(self, tokens: int) -> int:
        k = self.keep_activations
        if k == "auto":
            # Measured on the first step of a token count and reused after:
            # cudaMemGetInfo costs ~1 ms of host time and can wait behind the
            # queued work, which at a few micro-batches per GPU starves the
            # device of launches.
            cached = self._keep_cache.get(tokens)
            if cached is not None:
                return cached
            # free HBM plus what the caching allocator holds but does not use
            # (the previous step's kept activations come back to it)
            free, _ = torch.cuda.mem_get_info(self.device)
            free += torch.cuda.memory_reserved(self.device) - torch.cuda.memory_allocated(self.device)
            budget = self.keep_budget_fraction * free
            per = tokens * self.saved_bytes_per_token()
            k = max(0, min(int(budget // max(per, 1)), self.num_layers))
            self._keep_cache[tokens] = k
            return k
        return max(0, min(int(k), self.num_layers))

    def forward(self, h: torch.Tensor) -> List[torch.Tensor]:
        """h: [B, S, hidden] bf16 (B stacked micro-batches).  Returns the L+1
        boundary activations (activations[i] = hidden state before layer i)."""
        pe = self.position_embeddings(h.shape[1], h.dtype)
        acts = [h]
        self._graphs.clear()
        L = self.num_layers
        keep = self._layers_to_keep(h.shape[0] * h.shape[1])
        self.last_kept = keep
        self.scheduler.prefetch(0)
        for l in range(L):
            self.scheduler.prefetch(l + 1)
            self._load(l)
            chunks = self._chunks(h.shape[0])
            if l >= L - keep and len(chunks) == 1:
                x = h.detach().requires_grad_(True)
                with torch.enable_grad():
                    y = self.layer(x, position_embeddings=pe)
                self._graphs[l] = (x, y)
                out = y.detach()
            else:
                with torch.no_grad():
                    if len(chunks) == 1:
                        out = self.layer(h, position_embeddings=pe)
                    else:
                        out = torch.empty_like(h)
                        for a, b in chunks:
                            out[a:b] = self.layer(h[a:b], position_embeddings=pe)
            self.scheduler.release(l)
            h = out
            acts.append(h)
        return acts

    def backward(self, acts: Sequence[torch.Tensor], grad_out: torch.Tensor) -> torch.Tensor:
        """Reverse layer loop with recompute; accumulates LoRA grads into
        store.grad (caller zeroes it per optimizer step) and returns the
        gradient w.r.t. activations[0]."""
        pe = self.position_embeddings(grad_out.shape[1], grad_out.dtype)
        g = grad_out
        L = self.num_layers
        self.scheduler.prefetch(L - 1)
        for l in reversed(range(L)):
            self.scheduler.prefetch(l - 1)
            self._load(l)
            h_prev = acts[l]
            if l in self._graphs:  # forward kept its autograd state: no recompute
                x, y = self._graphs.pop(l)
                y.backward(g)
                g_in = x.grad
                del x, y
                self.scheduler.release(l)
                if self.comm is not None:
                    self.comm.allreduce_layer(l)
                g = g_in
                continue
            chunks = self._chunks(h_prev.shape[0])
            g_in = None if len(chunks) == 1 else torch.empty_like(h_prev)
            for a, b in chunks:
                x = h_prev[a:b].detach().requires_grad_(True)
                with torch.enable_grad():
                    y = self.layer(x, position_embeddings=pe)
                y.backward(g[a:b])
                if g_in is None:
                    g_in = x.grad
                else:
                    g_in[a:b] = x.grad
                del x, y
            self.scheduler.release(l)
            if self.comm is not None:
                self.comm.allreduce_layer(l)
            g = g_in
        if self.comm is not None:
            self.comm.wait()
        return g

    def step(self, h: torch.Tensor, grad_out: torch.Tensor) -> torch.Tensor:
        acts = self.forward(h)
        return self.backward(acts, grad_out)

    def step_with_loss(self, h: torch.Tensor, labels: torch.Tensor, head, grad_accum: int):
        """The reference's step (fitllm/trainer.py:495-535): forward over all
        layers, per micro-batch CE loss of the final norm + lm_head
        (``head``: lm_head.LMHeadLoss) scaled by 1/grad_accum, backward.
        Returns (per-micro-batch losses as device scalars, grad w.r.t. h)."""
        acts = self.forward(h)
        losses, grad_out = head.loss_and_grad_microbatches(acts[-1], labels, 1.0 / grad_accum)
        acts[-1] = None  # the last layer's output is only needed by the head
        return losses, self.backward(acts, grad_out)


def _lora_store(cfg: LayerConfig, num_layers: int, dev, seed: int, lora_b_std: float) -> LoRAStore:
    """LoRAStore with PEFT-initialised adapters per layer: A ~ U(-1/sqrt(K),
    1/sqrt(K)) (Kaiming-uniform, a=sqrt(5)); B zeros, or N(0, lora_b_std)."""
    proto = DecoderLayer(cfg, device="meta")
    add_lora_(proto, cfg.lora_rank, cfg.lora_alpha, cfg.lora_targets, seed=0)
    entries = lora_entries(proto)
    store = LoRAStore(num_layers, entries, dev)
    for l in range(num_layers):
        g = torch.Generator(device=dev).manual_seed(seed * 7919 + l)
        vals = {}
        for name, shape in entries:
            if "lora_A" in name:
                bound = 1.0 / (shape[1] ** 0.5)
                vals[name] = (torch.rand(shape, generator=g, device=dev) * 2 - 1) * bound
            elif lora_b_std > 0:
                vals[name] = torch.randn(shape, generator=g, device=dev) * lora_b_std
            else:
                vals[name] = torch.zeros(shape, device=dev)
        store.init_layer_(l, vals)
    return store


def synthetic_layer_shards(cfg: LayerConfig, num_layers: int, device, seed: int = 0):
    """Yields the flat shard key set of each random-init NF4 layer (quantised
    on the device with per-layer seeds seed * 1000 + l).  The tensors of one
    yield are overwritten by the next: consume (copy) each before advancing."""
    from .layer import quantize_layer_
    proto = DecoderLayer(cfg, device=torch.device(device))
    for l in range(num_layers):
        quantize_layer_(proto, seed=seed * 1000 + l)
        yield layer_shard(proto)
    del proto


def build_synthetic_model(cfg: LayerConfig, num_layers: int, device, seed: int = 0,
                          ring_slots: int = 2, pin_memory: bool = True, lora_b_std: float = 0.01):
    """Random-init NF4 layers (quantised on the device, per-layer seeds) loaded
    into a pinned host store, plus a LoRAStore with PEFT-initialised adapters
    (B ~ N(0, lora_b_std) so that dA is non-zero).  Returns (scheduler, store)."""
    dev = torch.device(device)
    sched = ShardScheduler(num_layers, dev, ring_slots=ring_slots, pin_memory=pin_memory)
    for l, shard in enumerate(synthetic_layer_shards(cfg, num_layers, dev, seed)):
        sched.add_layer(l, shard)
    store = _lora_store(cfg, num_layers, dev, seed, lora_b_std)
    torch.cuda.empty_cache()
    return sched, store


def build_model_from_shards(cfg: LayerConfig, shard_dir, num_layers: int, device,
                            group_size: int = 1, verify_checksums: bool = True, seed: int = 0,
                            ring_slots: int = 2, pin_memory: bool = True,
                            lora_b_std: float = 0.01):
    """The same (scheduler, store) pair from FitLLM-format shard files
    (``layer_{i:03d}_weights.safetensors`` + ``.sha256``): each file is
    checksummed and read once into the pinned host store; LoRA keys in the
    files are dropped as the reference does (fitllm/forward.py:733-734) and the
    adapters get the PEFT initialisation."""
    from .shards import load_shards_into
    dev = torch.device(device)
    sched = ShardScheduler(num_layers, dev, ring_slots=ring_slots, pin_memory=pin_memory)
    load_shards_into(sched, shard_dir, num_layers, group_size=group_size,
                     verify_checksums=verify_checksums)
    return sched, _lora_store(cfg, num_layers, dev, seed, lora_b_std)
