#!/usr/bin/env python
"""QLoRA layer fwd+bwd tokens/s on a Qwen2.5-32B-shaped layer (B200).

Workload (default, the headline configuration): one Qwen2.5-32B-shaped
decoder layer (hidden 5120, 40/8 heads x 128, MLP 27648, RMSNorm, RoPE 1e6),
all seven projections NF4 (blocksize 64, double-quantised absmax) from seeded
N(0, 0.02) weights, LoRA r=16 / alpha=32 on q_proj and v_proj; one
shard-stationary layer step = forward over the micro-batches (no autograd) +
recompute-with-autograd + backward (dX, dA, dB) + the per-layer LoRA gradient
all-reduce + global-norm clip + AdamW, over grad_accum = 16 micro-batches of
1 x 2048 tokens (token ids uniform over vocab 152064, seeded; embeddings
N(0, 0.02); upstream gradient N(0, 1) at the layer output).  The 16
micro-batches are split across the N GPUs (fixed total work: strong scaling).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl fitq|reference]

One JSON line on rank 0 (see the keys at the end of main()).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "QLoRA layer fwd+bwd tokens/s @Qwen2.5-32B shape"
UNIT = "tokens/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="fitq", choices=["fitq", "reference"])
    ap.add_argument("--microbatches", type=int, default=16)
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gemv", action="store_true")
    ap.add_argument("--cpu-seq", type=int, default=2048)
    ap.add_argument("--gemv-case", default=None,
                    help="N,K,M[,R]: run one NF4 GEMV shape and exit (a profiling target)")
    ap.add_argument("--attn-case", default=None,
                    help="B,H,KVH,T,prefix: run the verify attention on one shape and exit")
    ap.add_argument("--train-attn-case", default=None,
                    help="B,S,H,KVH: time the causal training attention (fwd, bwd) against SDPA and exit")
    ap.add_argument("--ce-case", default=None,
                    help="rows,vocab: run the cross-entropy kernel on one shape and exit")
    ap.add_argument("--qproj-case", action="store_true",
                    help="run only the q_proj QLoRA fwd+bwd (512 x 5120 x 5120, r=16) and exit")
    ap.add_argument("--decode-case", default=None,
                    help="layers,batch,drafts: run only the decode / verify pass and exit")
    ap.add_argument("--full-step", choices=["auto", "on", "off"], default="auto",
                    help="also time a full 64-layer step with shards streamed from pinned host "
                         "memory (each rank pins only its 1/N byte range of every layer)")
    return ap.parse_args()


def workload(a):
    return {"workload": "qwen2.5-32b-layer-shard-stationary-fwd-bwd", "layers": 1,
            "grad_accum_microbatches": a.microbatches, "seq_len": a.seq, "hidden": 5120,
            "heads": 40, "kv_heads": 8, "intermediate": 27648, "lora_rank": 16, "lora_alpha": 32,
            "lora_targets": ["q_proj", "v_proj"], "nf4_blocksize": 64, "double_quant": True,
            "parallelism": f"microbatch-dp{a.gpus}",
            "l2": "inputs larger than L2 (activations 335 MB per 16x2048 batch, weights 251.5 MB)"}


# Algorithmic FLOPs per token (no recompute counted): projections 4*P_layer
# (fwd 2P + dX 2P), LoRA 6r(N+K) for q and v, causal attention 3.5*2*S*d_model.
def flops_per_token(seq: int) -> float:
    p_layer = 487_587_840
    lora = 6 * 16 * (5120 + 5120) + 6 * 16 * (1024 + 5120)
    attn = 3.5 * 2 * seq * 5120
    return 4 * p_layer + lora + attn


class ClockSampler:
    """nvidia-smi clocks / throttle reasons around the timed region.

    Started before the warm-up and awaited until it writes its first sample,
    so that short timed regions (a few tens of ms at 8 GPUs) still see the
    GPU; samples are selected by their timestamps: those inside the timed
    window, else the last one before and the first one after it (the GPU is
    under the same load in the warm-up just before)."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None
        self.t0 = self.t1 = None

    def start(self, wait_s: float = 5.0):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return
        t_end = time.time() + wait_s
        while time.time() < t_end and os.path.getsize(self.path) == 0:
            time.sleep(0.02)

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()

    @staticmethod
    def _ts(field: str):
        import datetime
        try:
            return datetime.datetime.strptime(field.strip(), "%Y/%m/%d %H:%M:%S.%f").timestamp()
        except ValueError:
            return None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.12)  # one more sample after the window
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 10:
                rows.append((self._ts(f[0]), f[1:]))
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        inside = [r for t, r in rows if t is not None and self.t0 is not None and self.t0 <= t <= self.t1]
        sel, where = inside, "inside the timed region"
        if not sel:
            before = [r for t, r in rows if t is not None and self.t0 is not None and t < self.t0]
            after = [r for t, r in rows if t is not None and self.t1 is not None and t > self.t1]
            sel = before[-1:] + after[:1]
            where = "nearest before and after the timed region (shorter than the sampling period)"
        if not sel:
            sel, where = [r for _, r in rows], "whole run"
        sm = [float(r[1]) for r in sel if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in sel if r[2].replace(".", "").isdigit()]
        pw = [float(r[3]) for r in sel if r[3].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in sel for i in range(4) if r[5 + i].lower() == "active"})
        load = [v for v, w in zip(sm, pw) if w > 200] or sm
        return {"sm_mhz": statistics.median(load) if load else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(sel), "samples_from": where, "power_w_max": max(pw) if pw else None}


def cpu_baseline(a, seq):
    from oracle import layer_ref
    r = layer_ref.time_cpu_step(seq=seq, microbatches=1)
    return {"value": round(r["tokens_per_s"], 3), "unit": UNIT, "cores": r["threads"],
            "kind": "port",
            "sample": f"1 micro-batch x {seq} tokens through one layer step (fwd + recompute + bwd), "
                      f"fp32 torch CPU restatement with oracle-dequantised NF4 weights; "
                      f"{r['step_s']:.1f} s step (quantisation {r['quantize_s']:.1f} s untimed)"}


def gemv_sweep(dev, peak_gbs, reps=20, cpu=True):
    """NF4 GEMV decode sweep: HBM GB/s of the weight stream.

    Every shape rotates over enough distinct weights to exceed 2x L2, one
    pass over them is captured in a CUDA graph and replayed; time = CUDA
    events around the replays.  Bytes = packed NF4 + absmax codes + nested
    absmax of one weight per call."""
    import torch
    from fitllm_b200 import ops
    from fitllm_b200.nf4 import Nf4WeightCRef, quantize_nf4
    out = {}
    shapes = [("q_proj", 5120, 5120, 16), ("v_proj", 1024, 5120, 16), ("gate_up", 27648, 5120, 0),
              ("down", 5120, 27648, 0)]
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    g = torch.Generator(device=dev).manual_seed(11)
    for name, n, k, r in shapes:
        wbytes = n * k // 2 + n * k // 64 + ((n * k // 64 + 255) // 256) * 4
        nsets = max(2, int(2 * l2 // wbytes) + 1)
        sets = []
        for _ in range(nsets):
            w = torch.randn(n, k, generator=g, device=dev) * 0.02
            sets.append(Nf4WeightCRef(*quantize_nf4(w)))
            del w
        A = (torch.rand(r, k, generator=g, device=dev) - 0.5) * 0.02 if r else None
        B = torch.randn(n, r, generator=g, device=dev) * 0.01 if r else None
        for m in (1, 4, 16, 64):
            x = torch.randn(m, k, generator=g, device=dev).bfloat16()
            for wr in sets[:2]:
                ops.qlora_forward(x, wr, A, B, 2.0, gemv=True)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for wr in sets:
                    ops.qlora_forward(x, wr, A, B, 2.0, gemv=True)
            graph.replay()
            torch.cuda.synchronize()
            s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s_ev.record()
            for _ in range(reps):
                graph.replay()
            e_ev.record()
            torch.cuda.synchronize()
            us = s_ev.elapsed_time(e_ev) * 1000.0 / (reps * nsets)
            gbs = wbytes / (us * 1e-6) / 1e9
            out[f"{name}_{n}x{k}_m{m}"] = {"us": round(us, 2), "GB/s": round(gbs, 1),
                                          "frac_of_hbm": round(gbs / peak_gbs, 3),
                                          "lora": bool(r)}
            del graph
        del sets
        torch.cuda.empty_cache()
        if cpu:
            from oracle import layer_ref
            c = layer_ref.time_cpu_gemv(n, k, 1, r)
            out[f"{name}_{n}x{k}_m1"]["cpu_baseline"] = {
                "value": round(c["GB/s"], 3), "unit": "GB/s", "cores": c["threads"], "kind": "port",
                "sample": f"one M=1 call on the host cores: torch dequant in the oracle's op order + "
                          f"fp32 product ({c['us'] / 1000:.1f} ms)"}
    # The projections a decode layer issues together: q/k/v of one x as one
    # grouped call (LoRA on q and v) and gate/up with the SwiGLU applied
    # (fitq_nf4_gemv_grouped / fitq_nf4_gemv_swiglu): one GEMV launch and one
    # finishing launch each for M <= 8 (tcgen05 for larger M).
    for name, parts, swiglu in (("qkv_grouped", [(5120, 16), (1024, 0), (1024, 16)], False),
                                ("gate_up_swiglu", [(27648, 0), (27648, 0)], True)):
        k = 5120
        wbytes = sum(n * k // 2 + n * k // 64 + ((n * k // 64 + 255) // 256) * 4 for n, _ in parts)
        nsets = max(2, int(2 * l2 // wbytes) + 1)
        sets = []
        for _ in range(nsets):
            jobs = []
            for n, r in parts:
                w = torch.randn(n, k, generator=g, device=dev) * 0.02
                wr = Nf4WeightCRef(*quantize_nf4(w))
                del w
                A = (torch.rand(r, k, generator=g, device=dev) - 0.5) * 0.02 if r else None
                B = torch.randn(n, r, generator=g, device=dev) * 0.01 if r else None
                jobs.append((wr, A, B, 2.0, None, None))
            sets.append(jobs)
        for m in (1, 4, 16, 64):
            x = torch.randn(m, k, generator=g, device=dev).bfloat16()

            def call(jobs):
                if swiglu:
                    ops.nf4_gemv_swiglu(x, jobs[0], jobs[1])
                else:
                    ops.nf4_gemv_grouped(x, jobs)

            for jobs in sets[:2]:
                call(jobs)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for jobs in sets:
                    call(jobs)
            graph.replay()
            torch.cuda.synchronize()
            s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s_ev.record()
            for _ in range(reps):
                graph.replay()
            e_ev.record()
            torch.cuda.synchronize()
            us = s_ev.elapsed_time(e_ev) * 1000.0 / (reps * nsets)
            gbs = wbytes / (us * 1e-6) / 1e9
            out[f"{name}_m{m}"] = {"us": round(us, 2), "GB/s": round(gbs, 1),
                                   "frac_of_hbm": round(gbs / peak_gbs, 3),
                                   "weights": [f"{n}x{k}" + ("+lora" if r else "") for n, r in parts]}
            del graph
        del sets
        torch.cuda.empty_cache()
    return out


def qproj_linear(dev, reps=20, cpu=True):
    """BASELINE config 1 on the GPU: one NF4 QLoRA q_proj (5120 -> 5120, r=16,
    alpha 32) forward + backward (dX, dA, dB) over x [512, 5120] through the
    C-ABI calls (fitq_qlora_fwd / fitq_qlora_bwd), replayed from a CUDA graph
    with L2 flushed (a 256 MB write) before every replay; device time by CUDA
    events.  FLOPs per call = M (4 N K + 6 r (N + K)).  Also the same call
    through the module API (autograd, eager launches: host-launch bound at this
    size), and the CPU restatement."""
    import torch
    from fitllm_b200 import ops
    from fitllm_b200.qlora import Linear4bit, QLoRALinear4bit
    m, n, k, r = 512, 5120, 5120, 16
    g = torch.Generator(device=dev).manual_seed(0)
    w = torch.randn(n, k, generator=g, device=dev) * 0.02
    mod = QLoRALinear4bit(Linear4bit.from_float(w, None), r=r, lora_alpha=32.0).to(dev)
    del w
    with torch.no_grad():
        mod.lora_B["default"].weight.normal_(0.0, 0.01, generator=g)
    x = torch.randn(m, k, generator=g, device=dev).bfloat16().requires_grad_(True)
    dy = torch.randn(m, n, generator=g, device=dev).bfloat16()
    wref = mod.base_layer.wref()
    A = mod.lora_A["default"].weight.detach().float().contiguous()
    B = mod.lora_B["default"].weight.detach().float().contiguous()
    xd = x.detach()
    s = mod.scaling["default"]

    def abi_call():
        y, t = ops.qlora_forward(xd, wref, A, B, s, want_t=True)
        return ops.qlora_backward(xd, dy, wref, A, B, s, t_saved=t)

    for _ in range(3):
        abi_call()
    torch.cuda.synchronize()
    cs = torch.cuda.Stream(device=dev)
    cs.wait_stream(torch.cuda.current_stream(dev))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(cs):
        abi_call()
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=cs):
            abi_call()
    torch.cuda.synchronize()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    times = []
    for _ in range(reps):
        flush.zero_()
        s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s_ev.record()
        graph.replay()
        e_ev.record()
        torch.cuda.synchronize()
        times.append(s_ev.elapsed_time(e_ev))
    ms = statistics.median(times)
    del graph, flush

    def mod_call():
        mod.zero_grad(set_to_none=True)
        x.grad = None
        mod(x).backward(dy)

    for _ in range(3):
        mod_call()
    torch.cuda.synchronize()
    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_ev.record()
    for _ in range(reps):
        mod_call()
    e_ev.record()
    torch.cuda.synchronize()
    ms_mod = s_ev.elapsed_time(e_ev) / reps
    flops = m * (4 * n * k + 6 * r * (n + k))
    out = {"metric": "NF4 QLoRA q_proj fwd+bwd (x [512, 5120], r=16)", "ms": round(ms, 4),
           "tokens_per_s": round(m / (ms / 1000.0), 1),
           "tflops": round(flops / (ms / 1000.0) / 1e12, 1), "flop_per_call": flops,
           "timing": "C-ABI fwd + bwd replayed from a CUDA graph, L2 flushed before each replay, median of "
                     f"{reps}",
           "module_api_eager_ms": round(ms_mod, 4)}
    if cpu:
        from oracle import layer_ref
        c = layer_ref.time_cpu_qproj(m, n, k, r)
        out["cpu_baseline"] = {"value": round(c["tokens_per_s"], 1), "unit": "tokens/s",
                               "cores": c["threads"], "kind": "port",
                               "sample": f"the whole call (x [512, 5120]) in fp32 torch on the host "
                                         f"cores with the oracle-dequantised weight: "
                                         f"{c['call_s'] * 1000:.1f} ms per fwd+bwd"}
    return out


def nf4_layers(dev, layers_n=64):
    """64 random-init NF4 Qwen2.5-32B-shaped layers with LoRA r=16 on q/v."""
    from fitllm_b200.layer import DecoderLayer, LayerConfig, add_lora_, quantize_layer_
    cfg = LayerConfig.qwen25_32b()
    layers = []
    for i in range(layers_n):
        layer = DecoderLayer(cfg, device=dev)
        quantize_layer_(layer, seed=1000 + i)
        add_lora_(layer, cfg.lora_rank, cfg.lora_alpha, cfg.lora_targets, seed=i, b_std=0.01)
        layer.eval()
        layers.append(layer)
    return layers


def verify_bench(dev, peak_gbs, layers, batch=8, drafts=4, context=4096, reps=10, cpu=True):
    """one speculative-verify pass over 64 random-init NF4
    Qwen2.5-32B-shaped layers (LoRA r=16 on q/v), batch 8 x (4 draft + 1)
    tokens against a 4096-position KV cache -> every projection an M = 40 NF4
    GEMM; with batch 1 and no drafts, the single-token decode pass (every
    projection an M = 1 NF4 GEMV).  CUDA-graph replay; bytes = NF4 weights +
    KV read per pass."""
    import torch
    from fitllm_b200.layer import LayerConfig
    from fitllm_b200.verify import KVCache, verify_pass
    cfg = LayerConfig.qwen25_32b()
    t = drafts + 1
    layers_n = len(layers)
    cache = KVCache(layers_n, batch, cfg.kv_heads, cfg.head_dim, context + t, dev)
    cache.fill_random_(context, seed=3)
    g = torch.Generator(device=dev).manual_seed(4)
    h = (torch.randn(batch, t, cfg.hidden, generator=g, device=dev) * 0.02).bfloat16()
    verify_pass(layers, h, cache, context)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = verify_pass(layers, h, cache, context)
    graph.replay()
    torch.cuda.synchronize()
    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_ev.record()
    for _ in range(reps):
        graph.replay()
    e_ev.record()
    torch.cuda.synchronize()
    ms = s_ev.elapsed_time(e_ev) / reps
    wbytes = layers_n * (cfg.nf4_weights_per_layer() // 2 + cfg.nf4_weights_per_layer() // 64 +
                         4 * ((cfg.nf4_weights_per_layer() // 64 + 255) // 256))
    kv = cache.bytes_read(context + t)
    gbs = (wbytes + kv) / (ms / 1000.0) / 1e9
    del graph, out, cache
    torch.cuda.empty_cache()
    what = (f"speculative verify pass, {layers_n} NF4 layers, batch {batch} x {t} tokens, KV {context}"
            if t > 1 else f"single-token decode pass, {layers_n} NF4 layers, batch {batch}, KV {context}")
    out = {"metric": what,
           "ms_per_pass": round(ms, 3), "tokens_per_s": round(batch * t / (ms / 1000.0), 1),
           "bytes_per_pass": int(wbytes + kv), "GB/s": round(gbs, 1),
           "frac_of_hbm": round(gbs / peak_gbs, 3), "m_per_projection": batch * t,
           "note": "CUDA-graph replay; projections on the NF4 skinny GEMMs"
                   + (" (M <= 8: the decode GEMV kernel)" if batch * t <= 8 else "")
                   + ", attention on the split-KV verify kernel (fitq_verify_attention)"}
    if cpu:
        from oracle import layer_ref
        c = layer_ref.time_cpu_verify_layer(batch, t, context)
        out["cpu_baseline"] = {"value": round(c["tokens_per_s"], 3), "unit": "tokens/s",
                               "cores": c["threads"], "kind": "port",
                               "sample": f"one layer of the KV-cached verify step in fp32 torch on the "
                                         f"host cores ({c['layer_s'] * 1000:.1f} ms), extrapolated to "
                                         f"64 layers ({c['pass_s_64_layers']:.2f} s per pass)"}
    return out


def full_step_bench(dev, rank, world, layers_n=64, microbatches=16, seq=1024, steps=2, cpu=True):
    """One full synthetic training step over 64 random-init
    NF4 Qwen2.5-32B-shaped layers whose shards live in pinned host memory and
    stream through the device ring (sharded upload + NCCL all-gather when
    world > 1), 16 micro-batches of 1024 tokens split over the ranks, the loss
    of every micro-batch from the final norm + bf16 lm_head (vocab 152,064) +
    cross-entropy on the device, the per-layer LoRA-gradient all-reduce, then
    clip + AdamW on the q/v adapters.  Seeded token ids uniform over the
    vocabulary, embedded with a random bf16 table; labels are the ids shifted
    by one.  Device time per step (CUDA events, max over ranks)."""
    import torch
    from fitllm_b200.distributed import LoRAGradComm, barrier, max_over_ranks, microbatch_range
    from fitllm_b200.engine import ShardStationaryEngine, build_synthetic_model
    from fitllm_b200.layer import LayerConfig
    from fitllm_b200.lm_head import random_lm_head
    from fitllm_b200.optimizer import ShardOptimizer
    cfg = LayerConfig.qwen25_32b()
    sched, store = build_synthetic_model(cfg, layers_n, dev, seed=7)
    comm = LoRAGradComm(store)
    eng = ShardStationaryEngine(cfg, sched, store, dev, comm=comm)
    opt = ShardOptimizer(store)
    mb0, mb1 = microbatch_range(microbatches, rank, world)
    g = torch.Generator(device=dev).manual_seed(8)
    ids = torch.randint(0, cfg.vocab, (microbatches, seq + 1), generator=g, device=dev)[mb0:mb1]
    emb = (torch.randn(cfg.vocab, cfg.hidden, generator=g, device=dev) * 0.02).bfloat16()
    h0 = emb[ids[:, :seq]].contiguous()
    labels = ids[:, 1:].contiguous()
    del emb
    head = random_lm_head(cfg.hidden, cfg.vocab, dev, seed=9)
    losses = []

    def step():
        store.zero_grad()
        losses[:] = eng.step_with_loss(h0, labels, head, microbatches)[0]
        opt.step()

    step()
    barrier()
    torch.cuda.synchronize()
    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_ev.record()
    for _ in range(steps):
        step()
    e_ev.record()
    torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(s_ev.elapsed_time(e_ev) / steps, dev)
    h2d = sum(sched.upload_bytes(l) for l in range(layers_n))
    out = {"metric": "full 64-layer QLoRA training step tokens/s (16 x 1024 tokens, shards from host)",
           "value": round(microbatches * seq / (ms / 1000.0), 1), "unit": "tokens/s",
           "ms_per_step": round(ms, 1), "layers": layers_n,
           "model_tflops": round(microbatches * seq * layers_n * flops_per_token(seq) / (ms / 1000.0) / 1e12, 1),
           "model_tflops_incl_lm_head": round(microbatches * seq * (layers_n * flops_per_token(seq) +
                                                                    4 * cfg.hidden * cfg.vocab)
                                              / (ms / 1000.0) / 1e12, 1),
           "loss": {"mean_ce_rank0_last_step": round(float(torch.stack(losses).mean()), 4),
                    "note": "random-init model: about ln(152064) = 11.93"},
           "layers_kept_without_recompute": eng.last_kept,
           "h2d_shard_bytes_per_layer_pass_per_rank": int(h2d // layers_n),
           "pinned_host_bytes_per_rank": sched.host_bytes(),
           "note": "each layer's shard is uploaded in the forward and again in the backward "
                   "(two-slot ring); model_tflops counts the 64 layers (2.085 PFLOP per step), "
                   "the lm_head adds 2 GEMMs of 2 x 5120 x 152064 FLOP per token"}
    del eng, sched, store, opt, h0, labels, head
    torch.cuda.empty_cache()
    if cpu and rank == 0:
        from oracle import layer_ref
        c = layer_ref.time_cpu_step(seq=seq, microbatches=1)
        out["cpu_baseline"] = {"value": round(c["tokens_per_s"] / layers_n, 3), "unit": "tokens/s",
                               "cores": c["threads"], "kind": "port",
                               "sample": f"1 micro-batch x {seq} tokens through one layer step (fwd + "
                                         f"recompute + bwd) in fp32 torch on the host cores "
                                         f"({c['step_s']:.1f} s), extrapolated to {layers_n} layers "
                                         "(the lm_head and optimizer not counted)"}
    return out


def gemv_case(dev, spec):
    """One NF4 GEMV shape on its own ("N,K,M[,R]"): three warm calls, then 20
    timed ones on one weight (L2-resident when it fits: a profiling target, not
    a bench number).  Used to capture the decode kernels under ncu."""
    import torch
    from fitllm_b200 import ops
    from fitllm_b200.nf4 import Nf4WeightCRef, quantize_nf4
    n, k, m, r = (list(map(int, spec.split(","))) + [0])[:4]
    g = torch.Generator(device=dev).manual_seed(12)
    w = torch.randn(n, k, generator=g, device=dev) * 0.02
    wr = Nf4WeightCRef(*quantize_nf4(w))
    del w
    A = (torch.rand(r, k, generator=g, device=dev) - 0.5) * 0.02 if r else None
    B = torch.randn(n, r, generator=g, device=dev) * 0.01 if r else None
    x = torch.randn(m, k, generator=g, device=dev).bfloat16()
    for _ in range(3):
        ops.qlora_forward(x, wr, A, B, 2.0, gemv=True)
    torch.cuda.synchronize()
    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_ev.record()
    for _ in range(20):
        ops.qlora_forward(x, wr, A, B, 2.0, gemv=True)
    e_ev.record()
    torch.cuda.synchronize()
    if ops.device_status() != 0:
        raise RuntimeError("device status error in the GEMV case")
    return {"gemv_case": spec, "us_per_call": round(s_ev.elapsed_time(e_ev) * 1000.0 / 20, 2)}


def attn_case(dev, spec):
    """One verify-attention shape on its own ("B,H,KVH,T,prefix"): caches of
    prefix + T positions, three warm calls then 20 timed (a profiling target)."""
    import torch
    from fitllm_b200 import ops
    b, h, kvh, t, prefix = map(int, spec.split(","))
    g = torch.Generator(device=dev).manual_seed(13)
    q = torch.randn(b, t, h, 128, generator=g, device=dev).bfloat16()
    kc = torch.randn(b, kvh, prefix + t, 128, generator=g, device=dev).bfloat16()
    vc = torch.randn(b, kvh, prefix + t, 128, generator=g, device=dev).bfloat16()
    for _ in range(3):
        ops.verify_attention(q, kc, vc, prefix)
    torch.cuda.synchronize()
    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_ev.record()
    for _ in range(20):
        ops.verify_attention(q, kc, vc, prefix)
    e_ev.record()
    torch.cuda.synchronize()
    us = s_ev.elapsed_time(e_ev) * 1000.0 / 20
    kv = 2 * kc.numel() * 2
    return {"attn_case": spec, "us_per_call": round(us, 2), "kv_bytes": kv,
            "kv_GB/s": round(kv / us / 1e3, 1)}


def train_attn_case(dev, spec):
    """Causal GQA training attention on one shape ("B,S,H,KVH", head_dim 128):
    fitq_attention_fwd / _bwd against torch SDPA (cuDNN) on the same bf16
    tensors, three warm calls then 10 timed of each (CUDA events).  FLOPs in
    the flash-attention convention: causal forward 2*B*H*S*S*D (two GEMMs over
    half the score matrix), backward 2.5x that."""
    import torch
    import torch.nn.functional as F
    from fitllm_b200.layer_ops import attention_backward, attention_forward
    b, s, h, kvh = map(int, spec.split(","))
    g = torch.Generator(device=dev).manual_seed(15)
    q = torch.randn(b, s, h, 128, generator=g, device=dev).bfloat16()
    k = torch.randn(b, s, kvh, 128, generator=g, device=dev).bfloat16()
    v = torch.randn(b, s, kvh, 128, generator=g, device=dev).bfloat16()
    do = torch.randn(b, s, h, 128, generator=g, device=dev).bfloat16()
    fwd_flop = 2.0 * b * h * s * s * 128
    res = {"train_attn_case": spec, "fwd_gflop": round(fwd_flop / 1e9, 1)}

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s_ev.record()
        for _ in range(10):
            fn()
        e_ev.record()
        torch.cuda.synchronize()
        return s_ev.elapsed_time(e_ev) / 10

    o, lse = attention_forward(q, k, v)
    res["fitq_fwd_ms"] = round(timed(lambda: attention_forward(q, k, v)), 4)
    res["fitq_bwd_ms"] = round(timed(lambda: attention_backward(q, k, v, o, lse, do)), 4)
    qt, kt, vt = (t.transpose(1, 2).detach().requires_grad_(True) for t in (q, k, v))
    dot = do.transpose(1, 2)
    ot = F.scaled_dot_product_attention(qt, kt, vt, is_causal=True, enable_gqa=True)
    res["sdpa_fwd_ms"] = round(timed(lambda: F.scaled_dot_product_attention(
        qt, kt, vt, is_causal=True, enable_gqa=True)), 4)
    res["sdpa_bwd_ms"] = round(timed(lambda: torch.autograd.grad(ot, (qt, kt, vt), dot,
                                                                 retain_graph=True)), 4)
    for key in ("fitq", "sdpa"):
        res[key + "_fwd_tflops"] = round(fwd_flop / res[key + "_fwd_ms"] / 1e9, 1)
        res[key + "_bwd_tflops"] = round(2.5 * fwd_flop / res[key + "_bwd_ms"] / 1e9, 1)
    return res


def ce_case(dev, spec):
    """fitq_cross_entropy on its own ("rows,vocab"): bf16 logits, three warm
    calls then 20 timed on fresh copies (a profiling target)."""
    import torch
    from fitllm_b200 import _lib, ops
    rows, vocab = map(int, spec.split(","))
    g = torch.Generator(device=dev).manual_seed(14)
    logits = (torch.randn(rows, vocab, generator=g, device=dev) * 2).bfloat16()
    labels = torch.randint(0, vocab, (rows,), generator=g, device=dev)
    L = _lib.load()
    loss = torch.empty((), dtype=torch.float32, device=dev)
    nb = L.fitq_cross_entropy_workspace(rows)
    ws = torch.empty(nb, dtype=torch.uint8, device=dev)
    work = logits.clone()

    def call():
        _lib.check(L.fitq_cross_entropy(work.data_ptr(), labels.data_ptr(), rows, vocab, -100, 1.0,
                                        loss.data_ptr(), ws.data_ptr(), nb, ops._stream(dev)),
                   "fitq_cross_entropy")
    for _ in range(3):
        call()
    torch.cuda.synchronize()
    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_ev.record()
    for _ in range(20):
        call()  # gradients of gradients after the first call: same traffic and work
    e_ev.record()
    torch.cuda.synchronize()
    us = s_ev.elapsed_time(e_ev) * 1000.0 / 20
    return {"ce_case": spec, "us_per_call": round(us, 2),
            "GB/s_algorithmic": round(3 * logits.numel() * 2 / us / 1e3, 1)}


def run_reference(a):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    base = cpu_baseline(a, a.cpu_seq)
    vals = []
    from oracle import layer_ref
    import torch
    w = layer_ref.build_layer(seed=0)
    g = torch.Generator().manual_seed(5)
    h = torch.randn(1, a.cpu_seq, 5120, generator=g).bfloat16().float()
    go = torch.randn(1, a.cpu_seq, 5120, generator=g).bfloat16().float()
    for i in range(a.warmup + a.steps):
        t0 = time.perf_counter()
        layer_ref.layer_step(w, h, go)
        dt = time.perf_counter() - t0
        if i >= a.warmup:
            vals.append(a.cpu_seq / dt)
    v = statistics.median(vals)
    out = {"impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": UNIT,
           "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup,
           "ms_per_step": round(1000 * a.cpu_seq / v, 1), "higher_is_better": True,
           "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
           "config": dict(workload(a), sample_microbatches=1, sample_seq=a.cpu_seq),
           "cpu_baseline": {"kind": "port", "cores": base["cores"], "value": round(v, 3),
                            "unit": UNIT, "sample": base["sample"]},
           "e2e": {"value": round(v, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def main():
    a = parse()
    if a.impl == "reference":
        return run_reference(a)

    import torch
    from fitllm_b200 import _lib
    from fitllm_b200.distributed import (LoRAGradComm, barrier, init_from_env, max_over_ranks,
                                         microbatch_range)
    from fitllm_b200.engine import ShardStationaryEngine, build_synthetic_model
    from fitllm_b200.layer import LayerConfig
    from fitllm_b200.optimizer import ShardOptimizer

    rank, world = init_from_env()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    L = _lib.load()
    for case, fn in ((a.gemv_case, gemv_case), (a.attn_case, attn_case), (a.ce_case, ce_case),
                     (a.train_attn_case, train_attn_case)):
        if case:
            if rank == 0:
                print(json.dumps(fn(dev, case)), flush=True)
            return
    if a.qproj_case:
        print(json.dumps(qproj_linear(dev, cpu=False)), flush=True)
        return
    if a.decode_case:
        n_layers, batch, drafts = (int(v) for v in a.decode_case.split(","))
        pk_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
        hbm = json.load(open(pk_path)).get("hbm_gbs", 6650.0) if os.path.exists(pk_path) else 6650.0
        print(json.dumps(verify_bench(dev, hbm, nf4_layers(dev, n_layers), batch=batch, drafts=drafts,
                                      cpu=False)), flush=True)
        return

    cfg = LayerConfig.qwen25_32b()
    sched, store = build_synthetic_model(cfg, 1, dev, seed=0)
    comm = LoRAGradComm(store)
    eng = ShardStationaryEngine(cfg, sched, store, dev, comm=comm)
    opt = ShardOptimizer(store)

    mb0, mb1 = microbatch_range(a.microbatches, rank, world)
    nmb = mb1 - mb0
    # Inputs: token ids -> embeddings (seeded, identical across N), upstream grad N(0,1).
    g = torch.Generator(device=dev).manual_seed(5)
    ids = torch.randint(0, cfg.vocab, (a.microbatches, a.seq), generator=g, device=dev)
    g.manual_seed(6)
    emb = torch.randn(cfg.vocab, cfg.hidden, generator=g, device=dev, dtype=torch.bfloat16) * 0.02
    h0 = emb[ids[mb0:mb1]].contiguous()
    del emb, ids
    g.manual_seed(7)
    gout_all = torch.randn(a.microbatches, a.seq, cfg.hidden, generator=g, device=dev,
                           dtype=torch.bfloat16)
    gout = gout_all[mb0:mb1].contiguous()
    del gout_all
    torch.cuda.empty_cache()

    def step():
        store.zero_grad()
        eng.step(h0, gout)
        opt.step()

    clocks = ClockSampler(local)
    clocks.start()  # running through the warm-up, so a short timed region still has samples
    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    if _lib.load().fitq_get_device_status(1, None) != 0:
        raise RuntimeError("device status error after warm-up")

    L.fitq_timing_enable(4096)
    barrier()
    torch.cuda.synchronize()
    launches0 = L.fitq_launch_count()
    s_ev = torch.cuda.Event(enable_timing=True)
    e_ev = torch.cuda.Event(enable_timing=True)
    clocks.mark_start()
    s_ev.record()
    for _ in range(a.steps):
        step()
    e_ev.record()
    launches = L.fitq_launch_count() - launches0
    torch.cuda.synchronize()
    clocks.mark_end()
    barrier()
    clk = clocks.stop()
    ms_local = s_ev.elapsed_time(e_ev) / a.steps
    import ctypes
    nmax = 4096
    ms_arr = (ctypes.c_float * nmax)()
    fl_arr = (ctypes.c_double * nmax)()
    n_t = L.fitq_timing_read(ms_arr, fl_arr, nmax)
    L.fitq_timing_enable(0)
    gemm_ms = sum(ms_arr[i] for i in range(n_t))
    gemm_flops = sum(fl_arr[i] for i in range(n_t))
    ms = max_over_ranks(ms_local, dev)
    tokens = a.microbatches * a.seq
    value = tokens / (ms / 1000.0)
    kept = eng.last_kept

    # Same step with the reference's full recompute (no activations kept), for comparison.
    eng.keep_activations = 0
    step()
    barrier()
    torch.cuda.synchronize()
    s_r = torch.cuda.Event(enable_timing=True)
    e_r = torch.cuda.Event(enable_timing=True)
    s_r.record()
    for _ in range(a.steps):
        step()
    e_r.record()
    torch.cuda.synchronize()
    barrier()
    ms_rc = max_over_ranks(s_r.elapsed_time(e_r) / a.steps, dev)
    eng.keep_activations = "auto"

    # ---------------------------------------------------------------- e2e
    e2e = None
    if not a.no_e2e:
        from fitllm_b200.host_io import HostBatchPipeline
        h_host = h0.cpu().pin_memory()
        g_host = gout.cpu().pin_memory()
        gin_host = torch.empty_like(h_host).pin_memory()
        lora_host = torch.empty(store.per_layer, dtype=torch.float32).pin_memory()
        shard_bytes = sched.upload_bytes(0)  # this rank's share when the upload is sharded
        pipe = HostBatchPipeline(dev, [h_host, g_host])

        def e2e_step(bufs):
            store.zero_grad()
            gin = eng.step(bufs[0], bufs[1])
            opt.step()
            # The layer shard is uploaded from pinned host memory for every step:
            # the next step's upload is queued now, into the ring's other slot,
            # so it overlaps this step's work (as layer l + 1's upload overlaps
            # layer l in a multi-layer model).
            sched.invalidate()
            sched.prefetch(0)
            # a copy: the next step zeroes the gradient buffer while this one is read back
            return [gin, store.layer_slice(store.grad, 0).clone()]

        def e2e_run(n):
            pipe.run(e2e_step, [(h_host, g_host)] * n, [(gin_host, lora_host)] * n)

        e2e_run(2)
        sched.wait_uploads()
        barrier()
        torch.cuda.synchronize()
        s2 = torch.cuda.Event(enable_timing=True)
        e2 = torch.cuda.Event(enable_timing=True)
        s2.record()
        e2e_run(a.steps)
        sched.wait_uploads()  # the timed region holds one shard upload per step
        e2.record()
        torch.cuda.synchronize()
        barrier()
        ms_e2e = max_over_ranks(s2.elapsed_time(e2) / a.steps, dev)
        e2e = {"value": round(tokens / (ms_e2e / 1000.0), 1), "unit": UNIT,
               "h2d_bytes_per_step": int(shard_bytes + h_host.numel() * 2 + g_host.numel() * 2),
               "d2h_bytes_per_step": int(gin_host.numel() * 2 + lora_host.numel() * 4),
               "ms_per_step": round(ms_e2e, 3),
               "layers_kept_without_recompute": eng.last_kept,
               "shard_upload": "sharded: 1/G of the shard per rank over PCIe + NCCL all-gather"
                               if sched.shard_upload else "replicated",
               "note": "public API with pinned host buffers: layer shard H2D through the staging "
                       "ring, hidden states and upstream grad H2D, input grad and LoRA grads D2H, "
                       "every step inside the timed region; the batch copies run on their own "
                       "streams through fitllm_b200.host_io.HostBatchPipeline (next batch's H2D "
                       "and previous result's D2H overlap the step) and the next step's shard "
                       "upload goes into the ring's other slot while the step runs"}

    # every rank takes part in the full-step measurement (it has collectives)
    full_step = None
    if a.full_step in ("on", "auto"):
        del eng, sched, store, opt, h0, gout
        if e2e is not None:
            del h_host, g_host, gin_host, lora_host, pipe
        torch.cuda.empty_cache()
        full_step = full_step_bench(dev, rank, world, cpu=not a.no_cpu_baseline)

    if rank != 0:
        return
    peaks = {}
    pk_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(pk_path):
        peaks = json.load(open(pk_path))
    peak = peaks.get("bf16_tflops_sustained")
    peak_src = "of measured (bf16_tflops_sustained, kernel timed inside a long step)"
    if peak is None:
        peak, peak_src = 1400.0, "of fallback (sustained 1.4 PFLOP/s)"
    achieved = gemm_flops / (gemm_ms / 1000.0) / 1e12 if gemm_ms > 0 else None
    # DRAM read + write per GEMM launch: 509.1 MB measured by ncu over the 70
    # GEMM launches of the same step at 2 x 2048 tokens
    # (profiles/gemm_bf16_tn_dram_traffic_qwen25_32b_layer_2x2048.md), scaled
    # by the rows each launch processes (the traffic grows with M).
    traffic = 509.1e6 * (a.microbatches * a.seq) / (2 * 2048)
    out = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded NF4 weights, token ids, upstream grad)",
        "config": workload(a),
        "model_tflops": round(tokens * flops_per_token(a.seq) / (ms / 1000.0) / 1e12, 1),
        "value_recompute_every_layer": round(tokens / (ms_rc / 1000.0), 1),
        "ms_per_step_recompute_every_layer": round(ms_rc, 3),
        "recompute": {"layers_kept_without_recompute": kept, "layers": 1,
                      "note": "forward keeps its autograd state for the layers whose activations fit "
                              "the HBM budget, so their backward skips the recompute",
                      "value_recompute_every_layer": round(tokens / (ms_rc / 1000.0), 1),
                      "ms_per_step_recompute_every_layer": round(ms_rc, 3)},
        "roofline": {"bound": "tensor", "kernel": "gemm_bf16_tn (tcgen05: the cta_group::2 pair kernel, the one-CTA kernel for K >= 4N)",
                     "achieved": round(achieved, 1) if achieved else None, "peak": peak,
                     "unit": "TFLOP/s", "frac": round(achieved / peak, 3) if achieved else None,
                     "peak_source": peak_src, "traffic": round(traffic),
                     "traffic_unit": "bytes per launch (ncu dram__bytes_read.sum + write.sum at "
                                     "2 x 2048 tokens, scaled by the rows)",
                     "launches": n_t, "gemm_ms_per_step": round(gemm_ms / a.steps, 3),
                     "gemm_share_of_step": round(gemm_ms / a.steps / ms, 3)},
        "clocks": clk,
        "gpu_launches": int(launches),
        "e2e": e2e,
    }
    if world == 1 and not a.no_gemv:
        hbm = peaks.get("hbm_gbs", 6650.0)
        out["gemv"] = {"metric": "NF4 GEMV decode HBM GB/s (weight bytes / time, CUDA-graph replay, "
                                 "weights rotated over > 2x L2)", "peak_gbs": hbm,
                       "peak_source": "of measured (hbm_gbs)" if "hbm_gbs" in peaks else "of fallback",
                       "results": gemv_sweep(dev, hbm, cpu=not a.no_cpu_baseline)}
    if full_step is not None:
        out["full_step"] = full_step
    if world == 1 and not a.no_gemv:
        out["qproj_linear"] = qproj_linear(dev, cpu=not a.no_cpu_baseline)
        layers = nf4_layers(dev)
        hbm = peaks.get("hbm_gbs", 6650.0)
        out["verify"] = verify_bench(dev, hbm, layers, cpu=not a.no_cpu_baseline)
        out["decode"] = verify_bench(dev, hbm, layers, batch=1, drafts=0, cpu=not a.no_cpu_baseline)
        del layers
    if world == 1 and not a.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(a, a.cpu_seq)
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
    import torch.distributed as _dist
    if _dist.is_available() and _dist.is_initialized():
        _dist.destroy_process_group()
