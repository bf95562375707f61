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


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--cpu-sample-layers", type=int, default=2)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


# ---------------------------------------------------------------------------- CPU (reference formula)
PROJ_SHAPES = {"qkv": (3 * HIDDEN, HIDDEN), "o": (HIDDEN, HIDDEN), "gu": (2 * MLP, HIDDEN), "down": (HIDDEN, MLP)}


def cpu_layer_weights(seed):
    """Random-init bf16 projection weights of one decoder layer, N(0, 0.02), drawn on the host."""
    import torch
    g = torch.Generator().manual_seed(seed)
    return {name: (torch.randn(n, k, generator=g) * 0.02).bfloat16() for name, (n, k) in PROJ_SHAPES.items()}


class CpuLayer:
    """One decoder layer evaluated with the reference's CPU dequantize-and-matmul
    formula for every projection (reference tests/test_kernels.py:42-44:
    F.linear(activation_reference(x, a), q.float() * scale[:, None])) and fp32
    torch ops for norms, rotary embedding and attention.

    `weights` maps qkv / o / gu / down to bf16 [N, K] host tensors -- the same
    values the GPU model is built from when the two are compared."""

    def __init__(self, weights, tokens=TOKENS):
        import torch
        from oracle import oracle as O
        self.tokens = tokens
        self.w = {}
        for name, wt in weights.items():
            codes, scale = O.weight_codes(wt.float().numpy(), 4, 8)
            self.w[name] = O.dequant_weight(torch.from_numpy(codes), torch.from_numpy(scale))  # hoisted
        inv = 1.0 / (10000.0 ** (torch.arange(0, 128, 2, dtype=torch.float32) / 128))
        ang = torch.arange(tokens, dtype=torch.float32)[:, None] * inv[None, :]
        self.cos, self.sin = ang.cos(), ang.sin()

    def forward(self, x):
        import torch
        import torch.nn.functional as F
        from oracle import oracle as O

        T = self.tokens

        def norm(v):
            return v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + 1e-5)

        def rope(t):
            a, b = t[..., :64], t[..., 64:]
            c, s = self.cos[:, None, :], self.sin[:, None, :]
            return torch.cat([a * c - b * s, b * c + a * s], -1)

        h = norm(x)
        qkv = O.dequant_linear(h, self.w["qkv"], None, 8)
        q, k, v = qkv.split(HIDDEN, -1)
        q = rope(q.view(T, 32, 128)).transpose(0, 1)
        k = rope(k.view(T, 32, 128)).transpose(0, 1)
        v = v.view(T, 32, 128).transpose(0, 1)
        a = F.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(0, 1).reshape(T, HIDDEN)
        x = x + O.dequant_linear(a, self.w["o"], None, 8)
        gu = O.dequant_linear(norm(x), self.w["gu"], None, 8)
        g, u = gu.split(MLP, -1)
        return x + O.dequant_linear(F.silu(g) * u, self.w["down"], None, 8)


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
            "l2": "inputs larger than L2 (3.4 GB packed weights streamed per chunk, L2 126 MB)"}


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
    pa, as_ = ops.quantize_group64(x, 8)
    out = torch.empty(TOKENS, 3 * HIDDEN, device="cuda", dtype=torch.bfloat16)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

    def launch():
        ops.packed_linear(pa, as_, backend.packed_weight, backend.weight_scale, None, HIDDEN, 4, 8, out=out)

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
    return statistics.median(times) * 1e-3


def profile_traffic():
    f = ROOT / "profiles" / "gemm_w4a8_qkv_m600.json"
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
        gemm_s = dominant_gemm(torch, model)
        peak = int8_peak_tops(torch)
        ops_per_launch = 2 * TOKENS * HIDDEN * 3 * HIDDEN
        achieved = ops_per_launch / gemm_s / 1e12
        traffic = profile_traffic()
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
                         "kernel": "group64_gemm_kernel W4A8 M=600 K=4096 N=12288 (QKV)",
                         "peak_source": "torch._int_mm int8 8192^3, measured in this run (of measured)",
                         "gemm_us": round(gemm_s * 1e6, 2)},
            "cpu_baseline": cpu,
            "clocks": clock_info,
            "gpu_launches": launches_per_step * args.steps,
        }
        print(json.dumps(line), flush=True)
    policy.release()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return line


def main():
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
        return
    ours(args)


if __name__ == "__main__":
    main()
