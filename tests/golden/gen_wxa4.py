"""Generate the per-row A4 backend golden vectors (wxa4.npz) from the reference.

Run (CPU only, in a checkout that has the reference project):

    python tests/golden/gen_wxa4.py --reference <path to the Actune checkout>

What it runs, all from the reference package imported from that path, under
``TRITON_INTERPRET=1`` with the two libdevice calls replaced by their documented
IEEE semantics (``rint`` = round-half-even, ``div_rn`` = correctly rounded binary32
division), as in gen_tokenwise.py:

* ``actune.kernels.wxa4_native._quantize_rows_a4_kernel`` -- the per-row dynamic
  INT4 activation quantizer (packed nibbles, one fp32 scale per row);
* ``_unpack_a4_to_int8_kernel`` -- its sign extension to INT8 for W8A4;
* ``W2A4NativeLinear`` / ``W4A4NativeLinear`` / ``W8A4NativeLinear`` constructed on
  CPU (their codebooks, the nested W8 refinement and the packed buffers are plain
  torch);
* for W8A4, ``_w8a8_gemm_kernel`` on the sign-extended activations and the
  module's ``weight_int8``, writing an fp32 output buffer.

The W2A4 / W4A4 GEMM of the reference is a CUDA extension for sm_80
(native_s4_extension_kernel.cu) that cannot run here; for those two the file holds
the inputs, buffers and activation codes, and the tests compare against the
oracle's restatement of that kernel's epilogue.
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
from gen_tokenwise import _install_shim  # noqa: E402

SHAPES = [(1, 256, 64, True), (19, 512, 96, True), (40, 1024, 160, False)]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ACTUNE_REFERENCE", ""),
                    help="path of the reference Actune checkout (the folder holding actune/)")
    ap.add_argument("--out", default=str(HERE))
    args = ap.parse_args()
    if not args.reference or not (Path(args.reference) / "actune").is_dir():
        sys.exit("--reference must point at the reference checkout (folder containing actune/)")
    sys.path.insert(0, args.reference)
    _install_shim()
    import torch
    import triton
    import actune.kernels.wxa4_native as N4
    import actune.kernels.w8a8_triton as T8

    out = {}
    for w, cls in ((2, N4.W2A4NativeLinear), (4, N4.W4A4NativeLinear), (8, N4.W8A4NativeLinear)):
        for si, (m, k, n, with_bias) in enumerate(SHAPES):
            seed = 1000 + 100 * w + si
            g = torch.Generator().manual_seed(seed)
            lin = torch.nn.Linear(k, n, bias=with_bias)
            with torch.no_grad():
                lin.weight.copy_(torch.randn(n, k, generator=g) * 0.02)
                lin.weight[0, :3] = 0.0
                lin.weight[1, 5] = 0.5
                if with_bias:
                    lin.bias.copy_(torch.randn(n, generator=g) * 0.1)
                lin = lin.bfloat16()
            layer = cls(lin)
            x = torch.randn(m, k, generator=g).bfloat16() * 2
            cols = torch.randperm(k, generator=torch.Generator().manual_seed(seed))[: max(1, k // 100)]
            x[:, cols] *= 20
            if m > 2:
                x[2] = 0.0                       # all-zero row: scale at the 1e-8 floor
            packed = torch.empty(m, k // 2, dtype=torch.uint8)
            scale = torch.empty(m, dtype=torch.float32)
            N4._quantize_rows_a4_kernel[(m,)](x, packed, scale, in_features=k, BLOCK_K=256, num_warps=4)
            act = torch.empty(m, k, dtype=torch.int8)
            N4._unpack_a4_to_int8_kernel[(triton.cdiv(packed.numel(), 256),)](packed, act, packed.numel(),
                                                                               BLOCK=256, num_warps=4)
            key = f"w{w}_s{si}"
            if w == 8:
                res = torch.empty(m, n, dtype=torch.float32)
                bm, bn, bk, nw = T8._config_for(m)
                has_bias = bool(layer.bias.numel())
                bias = layer.bias if has_bias else layer.weight_scale
                T8._w8a8_gemm_kernel[(triton.cdiv(m, bm), triton.cdiv(n, bn))](
                    act, layer.weight_int8, scale, layer.weight_scale, bias, res, m, out_features=n, in_features=k,
                    has_bias=has_bias, BLOCK_M=bm, BLOCK_N=bn, BLOCK_K=bk, num_warps=nw)
                wbuf = layer.weight_int8.numpy()
                codes = layer.weight_int8.t().contiguous().numpy()
                acc = act.numpy().astype(np.int64) @ codes.astype(np.int64).T
                ref = (acc.astype(np.float32) * scale.numpy()[:, None]) * layer.weight_scale.numpy()[None, :]
                if has_bias:
                    ref = ref + layer.bias.numpy()[None, :]
                assert np.abs(ref - res.numpy()).max() <= 1e-3 * max(1.0, np.abs(ref).max()), (w, si)
                out[f"{key}_out"] = res.numpy()
            else:
                wbuf = layer.packed_weight.numpy()
                p = layer.packed_weight.to(torch.int16)
                if w == 4:
                    fields = [((p & 15) ^ 8) - 8, (((p >> 4) & 15) ^ 8) - 8]
                else:
                    fields = [(((p >> (2 * i)) & 3) ^ 2) - 2 for i in range(4)]
                codes = torch.stack(fields, -1).reshape(n, k).to(torch.int8).numpy()
            out[f"{key}_x"] = x.view(torch.int16).numpy().view(np.uint16)
            out[f"{key}_weight"] = lin.weight.detach().view(torch.int16).numpy().view(np.uint16)
            out[f"{key}_packed"] = packed.numpy()
            out[f"{key}_act"] = act.numpy()
            out[f"{key}_scale"] = scale.numpy()
            out[f"{key}_codes"] = codes
            out[f"{key}_wbuf"] = wbuf
            out[f"{key}_ws"] = layer.weight_scale.numpy()
            if layer.bias.numel():
                out[f"{key}_bias"] = layer.bias.numpy()
            print(key, "ok", flush=True)
    np.savez_compressed(Path(args.out) / "wxa4.npz", **out)
    print("wxa4.npz", len(out))


if __name__ == "__main__":
    main()
