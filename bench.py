#!/usr/bin/env python
"""Benchmark: ms per action chunk of the OpenVLA-OFT-shaped W4A8 backbone.

Workload (the one the headline metric is quoted on): a
random-init Llama-2-7B-shaped backbone (32 layers, hidden 4096, MLP 11008) on a
600-token call (512 vision + 32 prompt + 56 parallel-decoded action tokens),
every projection installed through ``install_bank`` as a group-64 W4A8 packed
linear (two binary switchable matrices), precision switched per call in the
order q00 -> q01 -> q11 -> q10 through ``GraphReplay`` (one CUDA graph per
configuration).  A step = one call = one action chunk.

Lines (one JSON line from rank 0):
* default: this repository's sm_100a path; ``value`` = device time per chunk
  (whole job: max-over-ranks time per step / chunks per step), ``e2e`` = the
  same through the public call with the pinned-host input copy and the
  action read-back inside the timed region, ``roofline`` for the dominant
  kernel (the W4A8 QKV GEMM, INT8-tensor bound at M = 600) against the INT8
  peak measured here with torch._int_mm, ``cpu_baseline`` = the reference's CPU
  dequantize-and-matmul formula on a bounded sample of layers.
* ``--impl reference``: the reference's CPU formula (the oracle port) on the
  host cores, each step one whole chunk (all 32 layers).

Multi-GPU: one process per GPU (torchrun), independent policy replicas, no
data-path collective; ``scaling`` = weak.
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
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "ms per action chunk (OpenVLA-OFT-shape W4A8)"
TOKENS, HIDDEN, MLP, LAYERS = 600, 4096, 11008, 32
WORKLOAD = ("config2: OpenVLA-OFT-shaped Llama-2-7B (32 layers, hidden 4096, MLP 11008), 600 tokens "
            "(512 vision + 32 prompt + 56 action), W4A8-average bank with two switchable matrices, "
            "q00/q01/q11/q10 cycled per call, CUDA graph per configuration")


# pi0.5-shaped policy (bench.py --config 3).
METRIC3 = "ms per action chunk (pi0.5-shape W4A4, prefix + 10 flow-matching steps)"
P3 = dict(prefix=304, horizon=50, action_dim=32, steps=10, layers=18, vlm_hidden=2048, vlm_mlp=16384,
          expert_hidden=1024, expert_mlp=4096, heads=8, kv_heads=1, head_dim=256)
WORKLOAD3 = ("config3: pi0.5-shaped policy, Gemma-2B-like VLM (18 layers, hidden 2048, 8 heads / 1 KV head x 256, "
             "MLP 16384) over 256 image + 48 text tokens, Gemma-300M-like action expert (width 1024, MLP 4096) "
             "through 10 flow-matching Euler steps over a 50 x 32 Gaussian noise chunk, W4A4-average bank with two "
             "switchable matrices, q00/q01/q11/q10 cycled per call, CUDA graph per step shape")


# serving (bench.py --config 4).
METRIC4 = "aggregate action chunks/s (pi0.5-shape serving, 16 environments per GPU, per-request precision routing)"
ENVS4 = 16
WORKLOAD4 = ("config4: one replica of the config-3 pi0.5-shaped W4A4 policy per GPU serving 16 independent "
             "environments (224x224x3 uint8 image + 14-dim N(0,1) state per request); each request's "
             "configuration chosen by a random depth<=5, 3-leaf selector tree over the 13 action-history "
             "features + state (C++ router) with a two-request minimum dwell; environments grouped by "
             "configuration into batches of 4/8/16, one CUDA graph per batch, step shape and configuration")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--cpu-sample-layers", type=int, default=2)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--config", type=int, choices=[0, 1, 2, 3, 4], default=2,
                    help="2: OFT-shaped W4A8 backbone (the headline metric); 0: one W4A8 linear; 1: the 180-case "
                         "precision sweep; 3: pi0.5-shaped W4A4 policy; 4: serving 16 environments per GPU")
    ap.add_argument("--markdown", default=None, help="config 1: also write the per-case table here")
    return ap.parse_args()


# ---------------------------------------------------------------------------- CPU (reference formula)
PROJ_SHAPES = {"qkv": (3 * HIDDEN, HIDDEN), "o": (HIDDEN, HIDDEN), "gu": (2 * MLP, HIDDEN), "down": (HIDDEN, MLP)}


def cpu_layer_weights(seed):
    """Random-init bf16 projection weights of one decoder layer, N(0, 0.02), drawn on the host."""
    import torch
    g = torch.Generator().manual_seed(seed)
    return {name: (torch.randn(n, k, generator=g) * 0.02).bfloat16() for name, (n, k) in PROJ_SHAPES.items()}


class CpuLayer:
    """One pre-norm decoder layer evaluated with the reference's CPU
    dequantize-and-matmul formula for every projection (reference
    tests/test_kernels.py:42-44: F.linear(activation_reference(x, a),
    q.float() * scale[:, None])) and fp32 torch ops for norms, rotary embedding,
    attention and the gated activation.  The norm weights of the random-init
    models are the identity, so the norms carry none.

    `weights` maps qkv / o / gu / down to bf16 [N, K] host tensors -- the same
    values the GPU model is built from when the two are compared.  Defaults: the
    OFT (Llama-2-7B) layer; the pi0.5 layers pass their Gemma shapes, `gemma`
    (tanh-GELU gate) and the rotary position offset of their tokens."""

    def __init__(self, weights, tokens=TOKENS, heads=32, kv_heads=32, head_dim=128, gemma=False, w_bits=4,
                 a_bits=8, rope_offset=0):
        import torch
        from oracle import oracle as O
        self.tokens, self.heads, self.kv_heads, self.head_dim = tokens, heads, kv_heads, head_dim
        self.gemma, self.a_bits = gemma, a_bits
        self.w = {}
        for name, wt in weights.items():
            codes, scale = O.weight_codes(wt.float().numpy(), w_bits, a_bits)
            self.w[name] = O.dequant_weight(torch.from_numpy(codes), torch.from_numpy(scale))  # hoisted
        self.mlp = self.w["down"].shape[1]
        half = head_dim // 2
        inv = 1.0 / (10000.0 ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
        ang = torch.arange(rope_offset, rope_offset + tokens, dtype=torch.float32)[:, None] * inv[None, :half]
        self.cos, self.sin = ang.cos(), ang.sin()

    def forward(self, x, past=None, store=None, causal=True):
        import torch
        import torch.nn.functional as F
        from oracle import oracle as O

        T, H, KV, D = self.tokens, self.heads, self.kv_heads, self.head_dim

        def norm(v):
            return v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + (1e-6 if self.gemma else 1e-5))

        def rope(t):
            a, b = t[..., : D // 2], t[..., D // 2:]
            c, s = self.cos[:, None, :], self.sin[:, None, :]
            return torch.cat([a * c - b * s, b * c + a * s], -1)

        qkv = O.dequant_linear(norm(x), self.w["qkv"], None, self.a_bits)
        q, k, v = qkv.split([H * D, KV * D, KV * D], -1)
        q = rope(q.view(T, H, D)).transpose(0, 1)
        k = rope(k.view(T, KV, D)).transpose(0, 1)
        v = v.view(T, KV, D).transpose(0, 1)
        if store is not None:
            store.append((k, v))
        if past is not None:
            k, v = torch.cat([past[0], k], 1), torch.cat([past[1], v], 1)
        if KV != H:
            k, v = k.repeat_interleave(H // KV, 0), v.repeat_interleave(H // KV, 0)
        a = F.scaled_dot_product_attention(q, k, v, is_causal=causal and past is None)
        x = x + O.dequant_linear(a.transpose(0, 1).reshape(T, H * D), self.w["o"], None, self.a_bits)
        gu = O.dequant_linear(norm(x), self.w["gu"], None, self.a_bits)
        g, u = gu.split(self.mlp, -1)
        act = F.gelu(g, approximate="tanh") if self.gemma else F.silu(g)
        return x + O.dequant_linear(act * u, self.w["down"], None, self.a_bits)


def cpu_chunk(layers, x0, n_layers=LAYERS):
    """One action chunk of the CPU formula: n_layers decoder layers, cycling `layers`."""
    x = x0
    for i in range(n_layers):
        x = layers[i % len(layers)].forward(x)
    return x


def cpu_sample(layers_in_sample, repeats=3, warmup=1):
    """Median seconds for `layers_in_sample` layers of the CPU formula."""
    import torch
    torch.set_num_threads(os.cpu_count() or 1)
    layers = [CpuLayer(cpu_layer_weights(100 + i)) for i in range(min(layers_in_sample, 2))]
    x0 = torch.randn(TOKENS, HIDDEN, generator=torch.Generator().manual_seed(1)).bfloat16().float()
    for _ in range(warmup):
        cpu_chunk(layers, x0, layers_in_sample)
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        cpu_chunk(layers, x0, layers_in_sample)
        times.append(time.perf_counter() - t0)
    return statistics.median(times)


def bench_config(world, layers=LAYERS):
    """The `config` object both arms print (identical keys and values)."""
    return {"workload": WORKLOAD, "tokens": TOKENS, "layers": layers, "parallelism": f"replicas x{world}",
            "l2": "inputs larger than L2 (3.4 GB of packed weights per chunk, 6.5 GB as the int8 codes the tile "
                  "GEMM reads; L2 126 MB)"}


def reference_arm(args):
    """The reference's CPU path (its dequantize-and-matmul formula, as the oracle port)
    on the host cores: every step is one whole action chunk, all 32 decoder layers
    (two weight sets cycled; each layer's ~0.8 GB of fp32 weights is far beyond the
    CPU caches, so the cycling changes nothing about the memory traffic)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    torch.set_num_threads(os.cpu_count() or 1)
    layers = [CpuLayer(cpu_layer_weights(100 + i)) for i in range(2)]
    x0 = torch.randn(TOKENS, HIDDEN, generator=torch.Generator().manual_seed(1)).bfloat16().float()
    for _ in range(args.warmup):
        cpu_chunk(layers, x0, args.layers)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_chunk(layers, x0, args.layers)
    ms_step = (time.perf_counter() - t0) / args.steps * 1e3
    line = {"impl": "reference", "metric": METRIC, "value": round(ms_step, 3), "unit": "ms",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 3),
            "ms_per_chunk": round(ms_step, 3), "chunks_per_step": 1,
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic (seeded random activations, random-init weights)",
            "config": bench_config(world, args.layers),
            "cpu_baseline": {"value": round(ms_step, 3), "unit": "ms", "cores": torch.get_num_threads(),
                             "kind": "port",
                             "sample": f"whole chunks: {args.layers} decoder layers per step (two weight sets "
                                       "cycled) of the reference's dequantize-and-matmul formula (oracle port), "
                                       f"{args.steps} timed steps after {args.warmup} warm-up"},
            "e2e": {"value": round(ms_step, 3), "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------- config 3 on the CPU
def pi05_cpu_weights(stack, seed):
    """bf16 projection weights of one pi0.5 VLM or action-expert layer, N(0, 0.02)."""
    import torch
    hidden = P3["vlm_hidden"] if stack == "vlm" else P3["expert_hidden"]
    mlp = P3["vlm_mlp"] if stack == "vlm" else P3["expert_mlp"]
    hd, h, kv = P3["head_dim"], P3["heads"], P3["kv_heads"]
    shapes = {"qkv": ((h + 2 * kv) * hd, hidden), "o": (hidden, h * hd), "gu": (2 * mlp, hidden),
              "down": (hidden, mlp)}
    g = torch.Generator().manual_seed(seed)
    return {n: (torch.randn(r, c, generator=g) * 0.02).bfloat16() for n, (r, c) in shapes.items()}


class Pi05Cpu:
    """The pi0.5-shaped chunk with the reference's CPU formula in every projection:
    the VLM over the prefix (keys and values kept per layer), then the frozen
    ten-step Euler loop over the action expert (actune/models/pi05.py:28-37).
    `vlm` / `expert` are lists of CpuLayer, cycled over the 18 layers."""

    def __init__(self, vlm, expert, seed=0):
        import torch
        self.vlm, self.expert = vlm, expert
        g = torch.Generator().manual_seed(seed)
        w, a = P3["expert_hidden"], P3["action_dim"]
        self.action_in = torch.randn(w, a, generator=g) * 0.02
        self.time_in = torch.randn(w, w, generator=g) * 0.02
        self.time_out = torch.randn(w, w, generator=g) * 0.02
        self.action_out = torch.randn(a, w, generator=g) * 0.02
        half = w // 2
        self.freqs = torch.exp(-torch.arange(half, dtype=torch.float32) * (torch.log(torch.tensor(10000.0)) / half))

    def chunk(self, embeds, noise, layers=P3["layers"]):
        import torch
        import torch.nn.functional as F
        cache = []
        x = embeds
        for i in range(layers):
            x = self.vlm[i % len(self.vlm)].forward(x, store=cache, causal=False)
        dt = torch.tensor(-1.0 / P3["steps"], dtype=torch.float32)
        time_ = torch.tensor(1.0, dtype=torch.float32)
        x_t = noise
        for _ in range(P3["steps"]):
            ang = time_ * self.freqs
            tvec = F.linear(F.silu(F.linear(torch.cat([ang.sin(), ang.cos()]), self.time_in)), self.time_out)
            h = F.linear(x_t, self.action_in) + tvec
            for i in range(layers):
                h = self.expert[i % len(self.expert)].forward(h, past=cache[i], causal=False)
            h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + 1e-6)
            x_t = x_t + dt * F.linear(h, self.action_out)
            time_ = time_ + dt
        return x_t


def pi05_cpu_model(weight_sets=2):
    kw = dict(heads=P3["heads"], kv_heads=P3["kv_heads"], head_dim=P3["head_dim"], gemma=True, w_bits=4, a_bits=4)
    vlm = [CpuLayer(pi05_cpu_weights("vlm", 200 + i), tokens=P3["prefix"], **kw) for i in range(weight_sets)]
    expert = [CpuLayer(pi05_cpu_weights("expert", 300 + i), tokens=P3["horizon"], rope_offset=P3["prefix"], **kw)
              for i in range(weight_sets)]
    return Pi05Cpu(vlm, expert)


def pi05_cpu_inputs():
    import torch
    g = torch.Generator().manual_seed(1)
    embeds = torch.randn(P3["prefix"], P3["vlm_hidden"], generator=g).bfloat16().float()
    noise = torch.randn(P3["horizon"], P3["action_dim"], generator=torch.Generator().manual_seed(0))
    return embeds, noise


def bench_config3(world):
    return {"workload": WORKLOAD3, "prefix_tokens": P3["prefix"], "action_tokens": P3["horizon"],
            "denoise_steps": P3["steps"], "parallelism": f"replicas x{world}",
            "l2": "inputs larger than L2 (1.15 GB packed weights streamed per chunk, L2 126 MB)"}


def reference_arm3(args):
    """Config 3 on the host cores: every step one whole chunk with the reference's
    CPU formula (VLM prefix + ten expert passes, two weight sets cycled per stack)."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    torch.set_num_threads(os.cpu_count() or 1)
    model = pi05_cpu_model()
    embeds, noise = pi05_cpu_inputs()
    for _ in range(args.warmup):
        model.chunk(embeds, noise)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        model.chunk(embeds, noise)
    ms = (time.perf_counter() - t0) / args.steps * 1e3
    line = {"impl": "reference", "metric": METRIC3, "value": round(ms, 3), "unit": "ms", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "ms_per_chunk": round(ms, 3),
            "chunks_per_step": 1, "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
            "dtype": "fp32", "data": "synthetic (seeded random prefix embeddings and noise, random-init weights)",
            "config": bench_config3(world),
            "cpu_baseline": {"value": round(ms, 3), "unit": "ms", "cores": torch.get_num_threads(), "kind": "port",
                             "sample": "whole chunks (18 VLM layers over 304 tokens + 10 x 18 expert layers over 50 "
                                       "tokens, two weight sets cycled per stack) of the reference's "
                                       "dequantize-and-matmul formula (oracle port)"},
            "e2e": {"value": round(ms, 3), "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------- GPU helpers
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.file, stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        self.file.flush()
        rows = []
        with open(self.file.name) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        loaded = [x for x in sm if x > 0.5 * (max(mx) if mx else 1)] or sm
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def int8_peak_tops(torch):
    a = torch.randint(-127, 127, (8192, 8192), dtype=torch.int8, device="cuda")
    b = torch.randint(-127, 127, (8192, 8192), dtype=torch.int8, device="cuda")
    for _ in range(3):
        torch._int_mm(a, b.t())
    best = float("inf")
    for _ in range(10):
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        s.record()
        torch._int_mm(a, b.t())
        e.record()
        e.synchronize()
        best = min(best, s.elapsed_time(e))
    del a, b
    return 2 * 8192 ** 3 / (best * 1e-3) / 1e12


def dominant_gemm(torch, model):
    """Average device time of the W4A8 QKV GEMM (M=600, K=4096, N=12288) with L2 flushed."""
    from actune_b200 import ops
    layer = model.layers[0].qkv_proj  # ResidentLinear
    backend = layer.backends["w4a8"]
    x = torch.randn(TOKENS, HIDDEN, device="cuda").bfloat16()
    bits, codes8 = backend.activation_format(TOKENS)
    pa, as_ = ops.quantize_group64(x, bits, codes8=codes8)
    out = torch.empty(TOKENS, 3 * HIDDEN, device="cuda", dtype=torch.bfloat16)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

    weight, w, a = backend.operands(TOKENS)  # the int8 codes when the runtime decoded them

    def launch():
        ops.packed_linear(pa, as_, weight, backend.weight_scale, None, HIDDEN, w, a, out=out)

    for _ in range(3):
        launch()
    times = []
    for _ in range(20):
        flush.zero_()
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        s.record()
        launch()
        e.record()
        e.synchronize()
        times.append(s.elapsed_time(e))
    del flush
    return statistics.median(times) * 1e-3, w


def profile_traffic(decoded):
    f = ROOT / "profiles" / ("gemm_w4a8_decoded_qkv_m600.json" if decoded else "gemm_w4a8_qkv_m600.json")
    if f.exists():
        try:
            return json.loads(f.read_text()).get("dram_bytes_per_launch")
        except (ValueError, OSError):
            return None
    return None


def ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))

    from actune_b200.graph import GraphReplay
    from actune_b200.harness import config_cycle, make_oft_policy
    from actune_b200.precision import precision_profile

    torch.manual_seed(1234 + rank)
    model, runtime = make_oft_policy(layers=args.layers, tokens=TOKENS, seed=rank)
    # shared_a8: the glue kernels hand each projection its packed input (one quantizer
    # pass per activation instead of a separate launch per projection).
    policy = GraphReplay(model.forward, runtime.modules, shared_a8=True, max_graphs=12)
    policy.enabled = True
    cycle = config_cycle()
    host_in = torch.randn(TOKENS, HIDDEN, generator=torch.Generator().manual_seed(7 + rank)).bfloat16().pin_memory()
    dev_in = host_in.to("cuda")
    host_out = torch.empty(8, 7, dtype=torch.float32).pin_memory()

    def step(i, e2e=False):
        with precision_profile(cycle[i % len(cycle)]), torch.inference_mode():
            if e2e:
                dev_in.copy_(host_in, non_blocking=True)
            out = policy(dev_in)
            if e2e:
                host_out.copy_(out, non_blocking=True)
        return out

    # Capture the four per-configuration graphs (setup, not timed), then warm up.
    for i in range(len(cycle)):
        step(i)
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()

    def timed(e2e):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        s.record()
        for i in range(args.steps):
            step(i, e2e)
            if e2e:
                torch.cuda.current_stream().synchronize()  # the caller reads the actions every call
                _ = float(host_out[0, 0])
        e.record()
        e.synchronize()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ms = torch.tensor([s.elapsed_time(e) / args.steps], device="cuda")
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        return float(ms.item())

    with ClockSampler(local) as clocks:
        ms_step = timed(False)
    ms_step_e2e = timed(True)
    clock_info = clocks.summary()

    line = None
    if rank == 0:
        gemm_s, gemm_w = dominant_gemm(torch, model)
        peak = int8_peak_tops(torch)
        ops_per_launch = 2 * TOKENS * HIDDEN * 3 * HIDDEN
        achieved = ops_per_launch / gemm_s / 1e12
        traffic = profile_traffic(gemm_w == 8)
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            secs = cpu_sample(args.cpu_sample_layers)
            import torch as _t
            cpu = {"value": round(secs / args.cpu_sample_layers * LAYERS * 1e3, 1), "unit": "ms",
                   "cores": _t.get_num_threads(), "kind": "port",
                   "sample": f"{args.cpu_sample_layers} of {LAYERS} layers (median of 3 after 1 warm-up) of "
                             "the reference's CPU dequantize-and-matmul formula, scaled to a 32-layer chunk"}
        launches_per_step = args.layers * 12 + 1
        line = {
            "metric": METRIC, "value": round(ms_step / world, 4), "unit": "ms", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic (seeded random token embeddings, random-init weights)",
            "ms_per_chunk": round(ms_step / world, 4), "chunks_per_step": world,
            "config": bench_config(world, args.layers),
            "e2e": {"value": round(ms_step_e2e / world, 4), "unit": "ms",
                    "h2d_bytes_per_step": host_in.numel() * host_in.element_size(),
                    "d2h_bytes_per_step": host_out.numel() * host_out.element_size()},
            "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1),
                         "unit": "TOP/s (int8)", "frac": round(achieved / peak, 4), "traffic": traffic,
                         "kernel": "group64_gemm_kernel W4A8 M=600 K=4096 N=12288 (QKV), "
                                   + ("weight codes read as int8 (decoded copy)" if gemm_w == 8 else "packed 4-bit weights"),
                         "peak_source": "torch._int_mm int8 8192^3, measured in this run (of measured)",
                         "gemm_us": round(gemm_s * 1e6, 2)},
            "cpu_baseline": cpu,
            "clocks": clock_info,
            "gpu_launches": launches_per_step * args.steps,
            "decoded_weight_bytes": runtime.decoded_bytes,
        }
        print(json.dumps(line), flush=True)
    policy.release()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return line


def dominant_gemm3(torch, model):
    """Device time of the pi0.5 VLM gate/up GEMM (W4A4, M=304, K=2048, N=32768), L2 flushed."""
    from actune_b200 import ops
    backend = model.vlm[0].gate_up_proj.backends["w4a4"]
    k, n, m = P3["vlm_hidden"], 2 * P3["vlm_mlp"], P3["prefix"]
    x = torch.randn(m, k, device="cuda").bfloat16()
    bits, codes8 = backend.activation_format(m)
    pa, as_ = ops.quantize_group64(x, bits, codes8=codes8)
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

    weight, w, a = backend.operands(m)

    def launch():
        ops.packed_linear(pa, as_, weight, backend.weight_scale, None, k, w, a, out=out)

    for _ in range(3):
        launch()
    times = []
    for _ in range(20):
        flush.zero_()
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        s.record()
        launch()
        e.record()
        e.synchronize()
        times.append(s.elapsed_time(e))
    return statistics.median(times) * 1e-3, 2 * m * n * k


def ours3(args):
    """Config 3 on the GPU: one step = one action chunk = the prefix graph plus ten
    replays of the denoise-step graph (one CUDA graph per step shape and precision
    configuration), precision cycled q00 -> q01 -> q11 -> q10 per chunk."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    from actune_b200.graph import GraphReplay
    from actune_b200.harness import config_cycle, make_pi05_policy, sample_pi05
    from actune_b200.precision import precision_profile

    torch.manual_seed(4321 + rank)
    model, runtime = make_pi05_policy(seed=rank)
    prefix_replay = GraphReplay(model.prefix, runtime.modules, shared_a8=True, max_graphs=12)
    step_replay = GraphReplay(model.denoise_step, runtime.modules, shared_a8=True, max_graphs=12)
    prefix_replay.enabled = step_replay.enabled = True
    cycle = config_cycle()
    g = torch.Generator().manual_seed(7 + rank)
    host_embeds = torch.randn(P3["prefix"], P3["vlm_hidden"], generator=g).bfloat16().pin_memory()
    host_noise = torch.randn(P3["horizon"], P3["action_dim"], generator=g).pin_memory()
    dev_embeds, dev_noise = host_embeds.to("cuda"), host_noise.to("cuda")
    host_out = torch.empty(P3["horizon"], P3["action_dim"]).pin_memory()

    def step(i, e2e=False):
        with precision_profile(cycle[i % len(cycle)]), torch.inference_mode():
            if e2e:
                dev_embeds.copy_(host_embeds, non_blocking=True)
                dev_noise.copy_(host_noise, non_blocking=True)
            out = sample_pi05(model, prefix_replay, step_replay, dev_embeds, dev_noise)
            if e2e:
                host_out.copy_(out, non_blocking=True)
        return out

    for i in range(len(cycle)):
        step(i)
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()

    def timed(e2e):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        s.record()
        for i in range(args.steps):
            step(i, e2e)
            if e2e:
                torch.cuda.current_stream().synchronize()
                _ = float(host_out[0, 0])
        e.record()
        e.synchronize()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ms = torch.tensor([s.elapsed_time(e) / args.steps], device="cuda")
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        return float(ms.item())

    with ClockSampler(local) as clocks:
        ms_step = timed(False)
    ms_step_e2e = timed(True)
    clock_info = clocks.summary()
    if rank == 0:
        gemm_s, gemm_ops = dominant_gemm3(torch, model)
        peak = int8_peak_tops(torch)
        achieved = gemm_ops / gemm_s / 1e12
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            torch.set_num_threads(os.cpu_count() or 1)
            cpu_model = pi05_cpu_model(weight_sets=1)
            embeds, noise = pi05_cpu_inputs()
            cpu_model.chunk(embeds, noise, layers=1)
            t0 = time.perf_counter()
            cpu_model.chunk(embeds, noise, layers=1)
            secs = time.perf_counter() - t0
            cpu = {"value": round(secs * P3["layers"] * 1e3, 1), "unit": "ms", "cores": torch.get_num_threads(),
                   "kind": "port",
                   "sample": "1 of 18 layers of each stack (the VLM prefix pass and ten expert passes) of the "
                             "reference's CPU dequantize-and-matmul formula, scaled x18 to a chunk"}
        launches = P3["layers"] * 11 + P3["steps"] * (P3["layers"] * 11 + 12)
        line = {
            "metric": METRIC3, "value": round(ms_step / world, 4), "unit": "ms", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
            "ms_per_chunk": round(ms_step / world, 4), "chunks_per_step": world,
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic (seeded random prefix embeddings and Gaussian noise, random-init weights)",
            "config": bench_config3(world),
            "e2e": {"value": round(ms_step_e2e / world, 4), "unit": "ms",
                    "h2d_bytes_per_step": host_embeds.numel() * 2 + host_noise.numel() * 4,
                    "d2h_bytes_per_step": host_out.numel() * 4},
            "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1),
                         "unit": "TOP/s (int8)", "frac": round(achieved / peak, 4), "traffic": None,
                         "kernel": "group64_gemm_kernel W4A4 M=304 K=2048 N=32768 (VLM gate/up)"
                                   + (", codes read as int8 (decoded weights and activations)"
                                      if model.vlm[0].gate_up_proj.backends["w4a4"].decoded_path(P3["prefix"])
                                      else ""),
                         "peak_source": "torch._int_mm int8 8192^3, measured in this run (of measured)",
                         "gemm_us": round(gemm_s * 1e6, 2)},
            "cpu_baseline": cpu, "clocks": clock_info, "gpu_launches": launches * args.steps,
            "decoded_weight_bytes": runtime.decoded_bytes,
        }
        print(json.dumps(line), flush=True)
    prefix_replay.release()
    step_replay.release()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def bench_config4(world):
    return {"workload": WORKLOAD4, "envs_per_gpu": ENVS4, "prefix_tokens": P3["prefix"],
            "denoise_steps": P3["steps"], "parallelism": f"replicas x{world}",
            "l2": "inputs larger than L2 (1.15 GB packed weights streamed per batch, L2 126 MB)"}


def ours4(args):
    """Config 4: one step = one request round for all 16 environments of the
    replica (routing, dwell, grouping, batched chunks, actions back to the host)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    from actune_b200.harness import Pi05Serving
    from actune_b200.router import PrecisionTree, random_selector_tree
    from actune_b200.serving import EnvRouter, groups_by_configuration

    torch.manual_seed(99 + rank)
    serving = Pi05Serving(envs=ENVS4, seed=rank)
    rng = np.random.default_rng(1000 + rank)
    pool = 4  # distinct image / state sets cycled over the requests
    host_images = torch.from_numpy(rng.integers(0, 256, (pool, ENVS4, 224, 224, 3), dtype=np.uint8)).pin_memory()
    host_states = torch.from_numpy(rng.standard_normal((pool, ENVS4, 14)).astype(np.float32)).pin_memory()
    dev_images = host_images.to("cuda")
    dev_states = host_states.to("cuda")
    host_actions = torch.empty(ENVS4, P3["horizon"], P3["action_dim"]).pin_memory()

    def round_(i, router, e2e):
        k = i % pool
        if e2e:
            img = dev_images[0]
            img.copy_(host_images[k], non_blocking=True)
            st = dev_states[0]
            st.copy_(host_states[k], non_blocking=True)
        else:
            img, st = dev_images[k], dev_states[k]
        configs = router.assign(host_states[k].numpy())
        for c, envs, size in groups_by_configuration(configs, serving.buckets):
            out = serving.chunk(("q00", "q01", "q11", "q10")[c], img, st, envs, size)
            host_actions[torch.as_tensor(envs)] = out.cpu()
        router.observe(host_actions.numpy())

    # Selector tree: three leaves over the action features and the state, with
    # thresholds at medians of the values a first request produces.
    probe = EnvRouter(PrecisionTree({"profile_index": 2}, 14), ENVS4)
    round_(0, probe, False)
    x = np.concatenate([probe.features, host_states[0].numpy()], 1)
    med = {f: (lambda v: (lambda r: v))(float(np.median(x[:, f]))) for f in range(27)}
    tree = PrecisionTree(random_selector_tree(np.random.default_rng(7), 14, leaves=3, thresholds=med), 14)
    router = EnvRouter(tree, ENVS4)
    # Capture every bucket x configuration graph once, then warm up.
    for c in ("q00", "q01", "q11", "q10"):
        for b in serving.buckets:
            serving.chunk(c, dev_images[0], dev_states[0], np.arange(b), b)
    for i in range(args.warmup):
        round_(i, router, False)
    torch.cuda.synchronize()

    def timed(e2e):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        s.record()
        for i in range(args.steps):
            round_(i, router, e2e)
        e.record()
        e.synchronize()
        if world > 1:
            dist.barrier()
        ms = torch.tensor([s.elapsed_time(e) / args.steps], device="cuda")
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        return float(ms.item())

    with ClockSampler(local) as clocks:
        ms_round = timed(False)
    ms_round_e2e = timed(True)
    clock_info = clocks.summary()
    if rank == 0:
        from actune_b200 import ops
        backend = serving.model.vlm[0].gate_up_proj.backends["w4a4"]
        m, k, n = ENVS4 * P3["prefix"], P3["vlm_hidden"], 2 * P3["vlm_mlp"]
        xq = torch.randn(m, k, device="cuda").bfloat16()
        bits, codes8 = backend.activation_format(m)
        pa, as_ = ops.quantize_group64(xq, bits, codes8=codes8)
        out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
        flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
        weight, w, a = backend.operands(m)
        times = []
        for r in range(13):
            flush.zero_()
            s, e = torch.cuda.Event(True), torch.cuda.Event(True)
            s.record()
            ops.packed_linear(pa, as_, weight, backend.weight_scale, None, k, w, a, out=out)
            e.record()
            e.synchronize()
            if r >= 3:
                times.append(s.elapsed_time(e) * 1e-3)
        gemm_s = statistics.median(times)
        peak = int8_peak_tops(torch)
        achieved = 2 * m * n * k / gemm_s / 1e12
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            torch.set_num_threads(os.cpu_count() or 1)
            cpu_model = pi05_cpu_model(weight_sets=1)
            embeds, noise = pi05_cpu_inputs()
            cpu_model.chunk(embeds, noise, layers=1)
            t0 = time.perf_counter()
            cpu_model.chunk(embeds, noise, layers=1)
            secs = (time.perf_counter() - t0) * P3["layers"]
            cpu = {"value": round(1.0 / secs, 4), "unit": "chunks/s", "cores": torch.get_num_threads(),
                   "kind": "port",
                   "sample": "one environment's chunk, 1 of 18 layers of each stack of the reference's CPU "
                             "dequantize-and-matmul formula timed and scaled x18 (environments served one "
                             "after another on the host cores)"}
        chunks_per_s = world * ENVS4 / (ms_round * 1e-3)
        line = {
            "metric": METRIC4, "value": round(chunks_per_s, 2), "unit": "chunks/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_round, 3),
            "chunks_per_step": world * ENVS4, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8", "data": "synthetic (uniform uint8 images, N(0,1) states, random-init weights)",
            "config": bench_config4(world),
            "e2e": {"value": round(world * ENVS4 / (ms_round_e2e * 1e-3), 2), "unit": "chunks/s",
                    "h2d_bytes_per_step": ENVS4 * (224 * 224 * 3 + 14 * 4),
                    "d2h_bytes_per_step": ENVS4 * P3["horizon"] * P3["action_dim"] * 4},
            "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1),
                         "unit": "TOP/s (int8)", "frac": round(achieved / peak, 4), "traffic": None,
                         "kernel": f"group64_gemm_kernel W4A4 M={m} K={k} N={n} (VLM gate/up, 16 environments)"
                                   + (", codes read as int8 (decoded weights and activations)"
                                      if backend.decoded_path(m) else ""),
                         "peak_source": "torch._int_mm int8 8192^3, measured in this run (of measured)",
                         "gemm_us": round(gemm_s * 1e6, 2)},
            "routing": {"switches": int(router.switches), "rounds": args.warmup + 2 * args.steps},
            "cpu_baseline": cpu, "clocks": clock_info,
            "decoded_weight_bytes": serving.runtime.decoded_bytes,
        }
        print(json.dumps(line), flush=True)
    serving.release()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def reference_arm4(args):
    """Config 4 on the host cores: the reference's CPU formula serves the
    environments one chunk at a time; each step is one environment's chunk."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    torch.set_num_threads(os.cpu_count() or 1)
    model = pi05_cpu_model()
    embeds, noise = pi05_cpu_inputs()
    for _ in range(args.warmup):
        model.chunk(embeds, noise)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        model.chunk(embeds, noise)
    secs = (time.perf_counter() - t0) / args.steps
    rate = 1.0 / secs
    line = {"impl": "reference", "metric": METRIC4, "value": round(rate, 4), "unit": "chunks/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(secs * 1e3, 3), "chunks_per_step": 1,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic (seeded random prefix embeddings and noise, random-init weights)",
            "config": bench_config4(world),
            "cpu_baseline": {"value": round(rate, 4), "unit": "chunks/s", "cores": torch.get_num_threads(),
                             "kind": "port", "sample": "one environment's whole chunk per step (reference's "
                                                       "dequantize-and-matmul formula, oracle port)"},
            "e2e": {"value": round(rate, 4), "unit": "chunks/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------- configs 0 and 1
_DEQUANT = {}


def cpu_formula_ms(m, k, n, w, a, threads, repeats=3):
    """Median ms of the reference's CPU dequantize-and-matmul formula for one linear
    (the weight dequantization hoisted and cached per shape and pair), on `threads`
    host threads."""
    import torch
    from oracle import oracle as O
    torch.set_num_threads(threads)
    key = (k, n, w, a)
    if key not in _DEQUANT:
        g = torch.Generator().manual_seed(k + n)
        wt = (torch.randn(n, k, generator=g) * 0.02).bfloat16().float()
        codes, scale = O.weight_codes(wt.numpy(), w, a)
        _DEQUANT.clear()  # one shape at a time keeps host memory bounded
        _DEQUANT[key] = O.dequant_weight(torch.from_numpy(codes), torch.from_numpy(scale))
    wd = _DEQUANT[key]
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(m)).bfloat16().float()
    O.dequant_linear(x, wd, None, a)
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        O.dequant_linear(x, wd, None, a)
        times.append((time.perf_counter() - t0) * 1e3)
    return statistics.median(times)


def config0(args):
    """one W4A8 linear, M=256, K=N=4096 (seed-0 recipe shapes):
    device time of the packed linear (L2 flushed, graph-replayed), the same call
    end to end from host buffers, and the CPU formula at all threads and at 1."""
    import torch
    from actune_b200 import ops
    from actune_b200.sweep import _graph_us, _int8_peak_tops
    m, k, n, w, a = 256, 4096, 4096, 4, 8
    torch.manual_seed(0)
    wt = (torch.randn(n, k) * 0.02).bfloat16().cuda()
    x = torch.randn(m, k)
    x[:, torch.randperm(k, generator=torch.Generator().manual_seed(0))[:41]] *= 20.0
    host_x = x.bfloat16().pin_memory()
    codes, ws = ops.weight_codes(wt, w, a)
    pw = ops.pack_rows(codes, w)
    dev_x = host_x.cuda()
    pa, as_ = ops.quantize_group64(dev_x, a)
    y = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
    us = _graph_us(lambda: ops.packed_linear(pa, as_, pw, ws, None, k, w, a, out=y), flush, 10)
    host_y = torch.empty(m, n, dtype=torch.bfloat16).pin_memory()
    workspace = torch.empty(ops.workspace_size(m, k, a), device="cuda", dtype=torch.uint8)

    def e2e_call():
        dev_x.copy_(host_x, non_blocking=True)
        ops.grouped_linear(dev_x, pw, ws, None, w, a, workspace=workspace, out=y)
        host_y.copy_(y, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    for _ in range(args.warmup):
        e2e_call()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_call()
    e2e_us = (time.perf_counter() - t0) / args.steps * 1e6
    peak = _int8_peak_tops(torch.device("cuda"))
    tops = 2 * m * n * k / us / 1e6
    cores = os.cpu_count() or 1
    cpu_all = cpu_formula_ms(m, k, n, w, a, cores)
    cpu_one = cpu_formula_ms(m, k, n, w, a, 1)
    print(json.dumps({
        "metric": "us per W4A8 linear (config 0: M=256, K=N=4096)", "value": round(us, 2), "unit": "us",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic (seed-0 recipe shapes, 41 outlier channels x20)",
        "config": {"workload": "config0: one group-64 W4A8 linear, M=256, K=N=4096, no bias",
                   "l2": "flushed between calls (64 Mi floats written)"},
        "e2e": {"value": round(e2e_us, 2), "unit": "us", "h2d_bytes_per_step": m * k * 2,
                "d2h_bytes_per_step": m * n * 2, "path": "actune_grouped_linear (quantize + GEMM)"},
        "roofline": {"bound": "tensor", "achieved": round(tops, 1), "peak": round(peak, 1), "unit": "TOP/s (int8)",
                     "frac": round(tops / peak, 4), "traffic": None},
        "cpu_baseline": {"value": round(cpu_all * 1e3, 1), "unit": "us", "cores": cores, "kind": "port",
                         "sample": "the whole linear (reference's dequantize-and-matmul formula, weights dequantized "
                                   "outside the timed region)", "one_thread_us": round(cpu_one * 1e3, 1)}}),
        flush=True)


def config1(args):
    """all nine pairs x four Llama projection shapes x M in
    {1, 8, 64, 256, 512}: device time per case (actune_b200.sweep: L2 flushed,
    graph-replayed) next to the CPU formula for the same case on all host threads
    (and on one thread for the single-token and 64-token cases)."""
    import torch
    from actune_b200 import sweep
    pairs = [(w, a) for w in (2, 4, 8) for a in (2, 4, 8)]
    ms = (1, 8, 64, 256, 512)
    result = sweep.run(pairs, ms, list(sweep.SHAPES), reps=10)
    cores = os.cpu_count() or 1
    cpu = {}
    for name, (k, n) in sweep.SHAPES.items():
        for (w, a) in pairs:
            for m in ms:
                cpu[(w, a, name, m)] = cpu_formula_ms(m, k, n, w, a, cores, repeats=1)
                if (w, a) == (4, 8):
                    cpu[("1t", name, m)] = cpu_formula_ms(m, k, n, 4, 8, 1, repeats=1) if m <= 64 else None
    total_gpu = sum(r["us"] for r in result["rows"])
    total_cpu = sum(cpu[(r["W"], r["A"], r["shape"], r["M"])] * 1e3 for r in result["rows"])
    for r in result["rows"]:
        r["cpu_us"] = round(cpu[(r["W"], r["A"], r["shape"], r["M"])] * 1e3, 1)
        one = cpu[("1t", r["shape"], r["M"])]
        r["cpu_1t_us_w4a8"] = None if one is None else round(one * 1e3, 1)
    if args.markdown:
        lines = [f"GPU: one B200, HBM peak {result['hbm_gbs']:.0f} GB/s (MEASURED_PEAKS.json), INT8 peak "
                 f"{result['int8_tops']:.0f} TOP/s (torch._int_mm 8192^3, same run).  CPU: the reference's "
                 f"dequantize-and-matmul formula on {cores} host threads (1-thread column: the W4A8 case).", "",
                 "| pair | shape | M | GPU us | of HBM | of INT8 | CPU us | CPU 1-thread us |",
                 "|---|---|---|---|---|---|---|---|"]
        for r in result["rows"]:
            lines.append(f"| W{r['W']}A{r['A']} | {r['shape']} | {r['M']} | {r['us']} | {r['hbm_frac']} | "
                         f"{r['int8_frac']} | {r['cpu_us']} | {r['cpu_1t_us_w4a8'] or ''} |")
        Path(args.markdown).write_text("\n".join(lines) + "\n")
    print(json.dumps({
        "metric": "us for the 180-case precision sweep (config 1, sum over cases)", "value": round(total_gpu, 1),
        "unit": "us", "n_gpus": 1, "steps": 1, "warmup": 3, "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic (random packed operands)",
        "config": {"workload": "config1: 9 pairs x {QKV, O, gate/up, down} x M in {1,8,64,256,512}",
                   "l2": "flushed before every call"},
        "cpu_baseline": {"value": round(total_cpu, 1), "unit": "us", "cores": cores, "kind": "port",
                         "sample": "every case once, the reference's dequantize-and-matmul formula"},
        "native_pairs_us": round(sum(r["us"] for r in result["rows"] if (r["W"], r["A"]) in NATIVE_PAIRS), 1),
        "hbm_gbs": result["hbm_gbs"], "int8_tops": result["int8_tops"], "cases": result["rows"]}), flush=True)


# The pairs the reference runs on its CUDA kernel (grouped_native.cu, W and A <= 4);
# pairs with an 8-bit operand run its Triton kernel.
NATIVE_PAIRS = ((2, 2), (2, 4), (4, 2), (4, 4))


def graph_time_us(torch, fn, flush, reps=10):
    """Per-call microseconds of fn() after an L2-evicting write: CUDA-graph replay of
    [flush, call] x reps minus that of [flush] x reps, CUDA events on the capturing
    stream, median of 5 replays."""
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        g_call, g_flush = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_call, stream=stream):
            for _ in range(reps):
                flush.zero_()
                fn()
        with torch.cuda.graph(g_flush, stream=stream):
            for _ in range(reps):
                flush.zero_()
    torch.cuda.synchronize()

    def replay(g):
        ts = []
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) * 1e3)
        return statistics.median(ts)

    us = (replay(g_call) - replay(g_flush)) / reps
    del g_call, g_flush
    return us


def config1_reference(args):
    """Reference arm of config 1: the reference's own GPU kernel for the pairs it
    runs natively -- grouped_native.cu's linear() (warp-level mma.sync int4, built
    from the reference's sources for sm_100a into oracle/_ref) -- on the config-1
    shapes and token counts, timed exactly as this library's sweep (L2 flushed,
    graph-replayed).  Its value is the sum over those 80 cases; this library's
    config-1 line carries the same sum as `native_pairs_us`."""
    import torch
    from oracle import build_ref
    ref = build_ref.load("ref_grouped_native")
    if ref is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/ref_grouped_native was not built (the "
                                                             "reference sources were absent at build time)"}))
        return
    dev = torch.device("cuda")
    flush = torch.empty(64 << 20, dtype=torch.float32, device=dev)
    shapes = {"qkv": (4096, 12288), "o": (4096, 4096), "gate_up": (4096, 22016), "down": (11008, 4096)}
    rows = []
    for (w, a) in NATIVE_PAIRS:
        for name, (k, n) in shapes.items():
            g = torch.Generator(device=dev).manual_seed(1000 * w + 10 * a + k + n)
            pw = torch.randint(0, 256, (n, k * w // 8), device=dev, dtype=torch.uint8, generator=g)
            ws = torch.rand(n, device=dev, generator=g) * 0.01
            bias = torch.empty(0, device=dev)
            for m in (1, 8, 64, 256, 512):
                pa = torch.randint(0, 256, (m, k * a // 8), device=dev, dtype=torch.uint8, generator=g)
                as_ = torch.rand(m, k // 64, device=dev, generator=g) * 0.01
                src = torch.empty(m, k, device=dev, dtype=torch.bfloat16)  # output dtype carrier
                us = graph_time_us(torch, lambda: ref.linear(pa, as_, pw, ws, bias, src, w, a), flush)
                rows.append({"W": w, "A": a, "shape": name, "M": m, "K": k, "N": n, "us": round(us, 2),
                             "tops": round(2 * m * n * k / us / 1e6, 1)})
    total = sum(r["us"] for r in rows)
    print(json.dumps({
        "impl": "reference", "metric": "us for the W{2,4}xA{2,4} cases of the config-1 sweep (sum over 80 cases)",
        "value": round(total, 1), "unit": "us", "n_gpus": 1, "steps": 1, "warmup": 3, "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "int4", "data": "synthetic (random packed operands)",
        "config": {"workload": "config1 native pairs: W{2,4}xA{2,4} x {QKV, O, gate/up, down} x M in "
                               "{1,8,64,256,512}", "l2": "flushed before every call"},
        "kernel": "reference grouped_native.cu linear() (mma.sync m16n8k64 s4), built from its sources for sm_100a",
        "e2e": {"value": round(total, 1), "unit": "us", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "cases": rows}), flush=True)


def main():
    args = parse()
    if args.config == 1 and args.impl == "reference":
        config1_reference(args)
        return
    if args.config in (0, 1):
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "config 0 is W4A8, which the reference runs on its "
                                                                 "Triton kernel (not built outside the reference "
                                                                 "tree); its CPU formula is the line's cpu_baseline"}),
                  flush=True)
            return
        (config0 if args.config == 0 else config1)(args)
        return
    if args.config == 3:
        (reference_arm3 if args.impl == "reference" else ours3)(args)
        return
    if args.config == 4:
        (reference_arm4 if args.impl == "reference" else ours4)(args)
        return
    if args.impl == "reference":
        reference_arm(args)
        return
    ours(args)


if __name__ == "__main__":
    main()
