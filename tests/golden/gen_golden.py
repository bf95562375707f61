"""Generate the golden vectors in this folder from the reference's own code.

Run (CPU only, in a checkout that has the reference project):

    python tests/golden/gen_golden.py --reference <path to the Actune checkout>

What it runs, all from the reference package imported from that path:

* ``actune.kernels.grouped._quantize_groups`` and ``_group_gemm`` -- the Triton
  kernels of the group-64 path -- under ``TRITON_INTERPRET=1``.  The two
  libdevice calls they make are replaced by their documented IEEE semantics:
  ``rint`` = round-half-even (``numpy.rint``) and ``div_rn`` = correctly rounded
  binary32 division (``numpy.divide`` on float32).  The GEMM writes an fp32
  output buffer: the interpreter's fp32->bf16 store truncates instead of
  rounding, so bf16 goldens would carry an interpreter artefact.
* ``actune.kernels.quantizers.weight_codes`` and ``actune.kernels.grouped.pack_rows``
  (plain torch, CPU) for the weight codebooks and their packing.
* ``actune.calibration.activation_reference`` as a cross-check of the
  interpreter's activation codes and scales.

Per-group int32 dots come from the same ``_group_gemm`` run one 64-wide group at
a time with unit scales, so they are the reference kernel's own integer dots.

Outputs (numpy .npz, a few hundred KB in total):
  quantize.npz   activation quantizer cases for A in {2,4,8}
  weights.npz    weight codes / scales / packed rows for all 9 pairs, with and
                 without per-row clip ratios
  gemm.npz       all 9 pairs x 3 shapes: inputs, packed operands, per-group
                 dots (first 8 rows for the largest shape) and the fp32 output
                 (with bias; one shape also without)
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402

HERE = Path(__file__).resolve().parent
PAIRS = [(w, a) for w in (2, 4, 8) for a in (2, 4, 8)]
GEMM_SHAPES = [(1, 64, 32), (17, 256, 96), (64, 1024, 64)]


def _install_shim(grouped):
    import triton.language as tl
    from triton.runtime.interpreter import TensorHandle

    def wrap(x, data):
        return tl.tensor(TensorHandle(np.asarray(data, dtype=np.float32), x.handle.dtype.scalar), x.type)

    class LibdeviceIEEE:
        @staticmethod
        def rint(x):
            return wrap(x, np.rint(x.handle.data))

        @staticmethod
        def div_rn(a, b):
            bd = b.handle.data if isinstance(b, tl.tensor) else np.float32(b)
            return wrap(a, np.divide(a.handle.data.astype(np.float32), np.asarray(bd, np.float32)))

    grouped.libdevice = LibdeviceIEEE


def _inputs(torch, m, k, seed, outlier_frac=0.01):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g)
    cols = torch.randperm(k, generator=torch.Generator().manual_seed(seed))[: max(1, int(k * outlier_frac))]
    x[:, cols] *= 20.0
    return x.bfloat16()


def _weight(torch, n, k, seed):
    g = torch.Generator().manual_seed(seed + 1000)
    w = torch.randn(n, k, generator=g) * 0.02
    w[0, :3] = 0.0          # a few structured values
    if n > 1:
        w[1, 5] = 0.5       # a row outlier
    return w.bfloat16()


def quantize_ref(torch, triton, G, x, a):
    m, k = x.shape
    packed = torch.empty((m, k * a // 8), dtype=torch.uint8)
    scales = torch.empty((m, k // 64), dtype=torch.float32)
    G._quantize_groups[(triton.cdiv(m * k // 64, 16),)](x.contiguous(), packed, scales, ELEMENTS=m * k, A=a,
                                                        num_warps=4)
    return packed, scales


def gemm_ref(torch, triton, G, packed, scales, pw, ws, bias, m, n, k, w, a):
    out = torch.empty((m, n), dtype=torch.float32)
    G._group_gemm[(triton.cdiv(m, 16), triton.cdiv(n, 32))](
        packed, pw, scales, ws, scales if bias is None else bias, out, m, N=n, K=k, W=w, A=a,
        BIAS=bias is not None, num_warps=4, num_stages=2)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ACTUNE_REFERENCE", ""),
                    help="path of the reference Actune checkout (the folder holding actune/)")
    ap.add_argument("--out", default=str(HERE))
    args = ap.parse_args()
    if not args.reference or not (Path(args.reference) / "actune").is_dir():
        sys.exit("--reference must point at the reference checkout (folder containing actune/)")
    sys.path.insert(0, args.reference)
    import torch
    import triton
    import actune.kernels.grouped as G
    from actune.kernels.quantizers import weight_codes
    from actune.calibration import activation_reference
    _install_shim(G)
    out = Path(args.out)

    # ---- activation quantizer -------------------------------------------------
    q = {}
    for a in (2, 4, 8):
        cases = []
        x0 = _inputs(torch, 17, 256, seed=a)
        x1 = _inputs(torch, 3, 64, seed=10 + a)
        x1[0] = 0.0                                   # all-zero group -> scale 1e-8/pos
        x1[1] = x1[1] * 1e-9                          # tiny values below the floor
        x1[2, :2] = torch.tensor([3.0, -3.0])         # ties around the grid
        x2 = _inputs(torch, 5, 128, seed=20 + a).float() * 3.0   # fp32 input case
        for i, x in enumerate((x0, x1, x2)):
            packed, scales = quantize_ref(torch, triton, G, x, a)
            # Cross-check against the reference's float codebook.
            deq = activation_reference(x, a).reshape(x.shape[0], -1, 64)
            s = scales.reshape(x.shape[0], -1, 1)
            assert torch.equal(deq, (deq / s).round() * s)
            q[f"a{a}_c{i}_x"] = (x.view(torch.int16).numpy().view(np.uint16) if x.dtype == torch.bfloat16
                                 else x.numpy())
            q[f"a{a}_c{i}_packed"] = packed.numpy()
            q[f"a{a}_c{i}_scales"] = scales.numpy()
    np.savez_compressed(out / "quantize.npz", **q)
    print("quantize.npz", len(q))

    # ---- weight codebooks -------------------------------------------------------
    wd = {}
    weight = _weight(torch, 96, 256, seed=3)
    clips = torch.linspace(0.7, 1.0, 96)
    wd["weight"] = weight.view(torch.int16).numpy().view(np.uint16)
    wd["clips"] = clips.numpy()
    for w, a in PAIRS:
        for tag, clip in (("noclip", None), ("clip", clips)):
            codes, scale = weight_codes(weight, w, a, clip_ratios=clip)
            wd[f"w{w}a{a}_{tag}_codes"] = codes.numpy()
            wd[f"w{w}a{a}_{tag}_scale"] = scale.numpy()
            wd[f"w{w}a{a}_{tag}_packed"] = G.pack_rows(codes, w).numpy()
    np.savez_compressed(out / "weights.npz", **wd)
    print("weights.npz", len(wd))

    # ---- GEMM -----------------------------------------------------------------
    gd = {}
    for si, (m, k, n) in enumerate(GEMM_SHAPES):
        x = _inputs(torch, m, k, seed=100 + si)
        weight = _weight(torch, n, k, seed=200 + si)
        bias_bf16 = (torch.randn(n, generator=torch.Generator().manual_seed(300 + si)) * 0.1).bfloat16()
        gd[f"s{si}_x"] = x.view(torch.int16).numpy().view(np.uint16)
        gd[f"s{si}_weight"] = weight.view(torch.int16).numpy().view(np.uint16)
        gd[f"s{si}_bias"] = bias_bf16.view(torch.int16).numpy().view(np.uint16)
        for w, a in PAIRS:
            key = f"s{si}_w{w}a{a}"
            codes, ws = weight_codes(weight, w, a)
            pw = G.pack_rows(codes, w)
            packed, scales = quantize_ref(torch, triton, G, x, a)
            bias = bias_bf16.float() if a == 4 else bias_bf16
            y = gemm_ref(torch, triton, G, packed, scales, pw, ws, bias.float(), m, n, k, w, a)
            gd[f"{key}_pw"] = pw.numpy()
            gd[f"{key}_ws"] = ws.numpy()
            gd[f"{key}_pa"] = packed.numpy()
            gd[f"{key}_as"] = scales.numpy()
            gd[f"{key}_y"] = y.numpy()
            if si == 1:
                gd[f"{key}_y_nobias"] = gemm_ref(torch, triton, G, packed, scales, pw, ws, None,
                                                  m, n, k, w, a).numpy()
            dots = np.zeros((m, n, k // 64), np.int32)
            ones_m = torch.ones((m, 1), dtype=torch.float32)
            ones_n = torch.ones((n,), dtype=torch.float32)
            for g in range(k // 64):
                pa_g = packed[:, g * 64 * a // 8:(g + 1) * 64 * a // 8].contiguous()
                pw_g = pw[:, g * 64 * w // 8:(g + 1) * 64 * w // 8].contiguous()
                yg = gemm_ref(torch, triton, G, pa_g, ones_m, pw_g, ones_n, None, m, n, 64, w, a)
                dots[:, :, g] = yg.numpy().astype(np.int32)
                assert np.array_equal(dots[:, :, g].astype(np.float32), yg.numpy())
            # The largest shape keeps the per-group dots of its first 8 rows
            # only (fixture size); its full output is still pinned by y.
            gd[f"{key}_dots"] = dots if si < 2 else dots[:8]
        print("gemm shape", (m, k, n), "done", flush=True)
    np.savez_compressed(out / "gemm.npz", **gd)
    print("gemm.npz", len(gd))


if __name__ == "__main__":
    main()
