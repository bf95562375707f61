"""Precision sweep of the packed linear (the reference's benchmark configuration 1).

    python -m actune_b200.sweep [--pairs 4x8,8x8] [--ms 1,8,64,256,512] [--json out.jsonl]

All nine W x A pairs in {2, 4, 8}^2 over the Llama-2-7B projection shapes (fused
QKV 4096 -> 12288, O 4096 -> 4096, fused gate/up 4096 -> 22016, down 11008 ->
4096) at M in {1, 8, 64, 256, 512} tokens, each timed through the public entry
point (`ops.packed_linear`, variant AUTO, bf16 output) on inputs resident in HBM.
Every call is preceded by a write of a 256 MiB buffer, which evicts the 126 MB L2,
and the per-call time is the CUDA-graph replay time of [flush, call] x R minus
that of [flush] x R (CUDA events on the capturing stream).  Reported per case:
microseconds, algorithmic bytes / time against the measured HBM copy bandwidth,
and int ops / time against the INT8 tensor peak measured in the same run with
`torch._int_mm` (8192^3).  Operand values are random bytes: the kernels' timing
does not depend on them (bit-exactness is the tests' job).
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import torch

from . import ops

SHAPES = {"qkv": (4096, 12288), "o": (4096, 4096), "gate_up": (4096, 22016), "down": (11008, 4096)}


def _hbm_peak_gbs() -> float:
    p = Path(__file__).resolve().parent.parent / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"])
    except (OSError, ValueError, KeyError):
        return 6650.0  # earlier measurement on the same pool, used when the file is absent


def _int8_peak_tops(dev) -> float:
    a = torch.randint(-128, 128, (8192, 8192), device=dev, dtype=torch.int8)
    b = torch.randint(-128, 128, (8192, 8192), device=dev, dtype=torch.int8)
    for _ in range(3):
        torch._int_mm(a, b.t())
    best = float("inf")
    for _ in range(5):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._int_mm(a, b.t())
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1) * 1e-3)
    return 2 * 8192 ** 3 / best / 1e12


def _graph_us(fn, flush, reps: int) -> float:
    """Per-call microseconds of fn() after an L2-evicting write, graph-replayed."""
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
        g.replay()
        torch.cuda.synchronize()
        ts = []
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) * 1e3)
        return sorted(ts)[2]

    us = (replay(g_call) - replay(g_flush)) / reps
    del g_call, g_flush
    return us


def run(pairs, ms, shapes, reps: int = 10, out=None):
    dev = torch.device("cuda", torch.cuda.current_device())
    hbm = _hbm_peak_gbs()
    int8 = _int8_peak_tops(dev)
    flush = torch.empty(64 << 20, dtype=torch.float32, device=dev)
    rows = []
    for (w, a) in pairs:
        for name in shapes:
            k, n = SHAPES[name]
            g = torch.Generator(device=dev).manual_seed(1000 * w + 10 * a + k + n)
            pw = torch.randint(0, 256, (n, k * w // 8), device=dev, dtype=torch.uint8, generator=g)
            ws = torch.rand(n, device=dev, generator=g) * 0.01
            for m in ms:
                pa = torch.randint(0, 256, (m, k * a // 8), device=dev, dtype=torch.uint8, generator=g)
                as_ = torch.rand(m, k // 64, device=dev, generator=g) * 0.01
                y = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
                us = _graph_us(lambda: ops.packed_linear(pa, as_, pw, ws, None, k, w, a, out=y), flush, reps)
                nbytes = n * k * w // 8 + m * k * a // 8 + 4 * m * (k // 64) + 4 * n + 2 * m * n
                tops = 2 * m * n * k / us / 1e6
                gbs = nbytes / us / 1e3
                row = {"W": w, "A": a, "shape": name, "M": m, "K": k, "N": n, "us": round(us, 2),
                       "GBps": round(gbs, 1), "hbm_frac": round(gbs / hbm, 3), "TOPS": round(tops, 1),
                       "int8_frac": round(tops / int8, 3)}
                rows.append(row)
                line = json.dumps(row)
                print(line, flush=True)
                if out is not None:
                    out.write(line + "\n")
    return {"hbm_gbs": hbm, "int8_tops": round(int8, 1), "rows": rows}


def markdown(result) -> str:
    lines = [f"HBM peak {result['hbm_gbs']:.0f} GB/s (MEASURED_PEAKS.json), INT8 peak {result['int8_tops']:.0f} "
             "TOP/s (torch._int_mm, same run).", "",
             "| pair | shape | M | us | GB/s | of HBM | TOP/s | of INT8 |", "|---|---|---|---|---|---|---|---|"]
    for r in result["rows"]:
        lines.append(f"| W{r['W']}A{r['A']} | {r['shape']} | {r['M']} | {r['us']} | {r['GBps']} | {r['hbm_frac']} | "
                     f"{r['TOPS']} | {r['int8_frac']} |")
    return "\n".join(lines)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--pairs", default="all", help="comma list like 4x8,8x8 (W x A), or 'all'")
    ap.add_argument("--ms", default="1,8,64,256,512")
    ap.add_argument("--shapes", default="qkv,o,gate_up,down")
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--json", default=None, help="also write JSON lines here")
    ap.add_argument("--markdown", default=None, help="also write a markdown table here")
    args = ap.parse_args(argv)
    if not torch.cuda.is_available():
        sys.exit("the sweep needs a CUDA device")
    if args.pairs == "all":
        pairs = [(w, a) for w in (2, 4, 8) for a in (2, 4, 8)]
    else:
        pairs = [tuple(int(v) for v in p.split("x")) for p in args.pairs.split(",")]
    ms = [int(v) for v in args.ms.split(",")]
    shapes = args.shapes.split(",")
    out = open(args.json, "w") if args.json else None
    try:
        result = run(pairs, ms, shapes, args.reps, out)
    finally:
        if out is not None:
            out.close()
    if args.markdown:
        Path(args.markdown).write_text(markdown(result) + "\n")


if __name__ == "__main__":
    main()
