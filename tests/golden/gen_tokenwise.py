"""Generate the tokenwise-backend golden vectors (tokenwise.npz) from the reference.

Run (CPU only, in a checkout that has the reference project):

    python tests/golden/gen_tokenwise.py --reference <path to the Actune checkout>

What it runs, all from the reference package imported from that path, under
``TRITON_INTERPRET=1`` with the two libdevice calls replaced by their documented
IEEE semantics (``rint`` = round-half-even, ``div_rn`` = correctly rounded binary32
division), as in gen_golden.py:

* ``actune.kernels.w4a8_triton._quantize_rows_kernel`` -- the fused per-row
  dynamic INT8 activation quantizer shared by the W4A8 / W8A8 / W2A8 modules;
* ``W4A8TritonLinear`` / ``W8A8TritonLinear`` / ``W2A8TritonLinear`` constructed
  on CPU (their weight codebooks and K-major packed buffers are plain torch);
* ``_w4a8_gemm_kernel`` / ``_w8a8_gemm_kernel`` / ``_w2a8_gemm_kernel`` on those
  buffers, writing an fp32 output buffer (the interpreter's fp32->bf16 store
  truncates instead of rounding).

Outputs (numpy .npz): per (W, shape) the bf16 input and weight bits, the activation codes
and row scales, the weight codes [N, K], the module's packed weight buffer and
row scales, the bf16 bias bits (or none) and the fp32 output.
"""
from __future__ import annotations

import argparse
import importlib
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402

HERE = Path(__file__).resolve().parent
SHAPES = [(1, 256, 64, True), (19, 512, 96, True), (40, 1024, 160, False)]


def _install_shim():
    import triton.language as tl
    import triton.language.extra as extra
    from triton.runtime.interpreter import TensorHandle

    def wrap(x, data):
        return tl.tensor(TensorHandle(np.asarray(data, dtype=np.float32), x.handle.dtype.scalar), x.type)

    lib = importlib.import_module("triton.language.extra.libdevice")
    lib.rint = lambda x: wrap(x, np.rint(x.handle.data))

    def div_rn(a, b):
        bd = b.handle.data if isinstance(b, tl.tensor) else np.float32(b)
        return wrap(a, np.divide(a.handle.data.astype(np.float32), np.asarray(bd, np.float32)))

    lib.div_rn = div_rn
    extra.libdevice = lib


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
    import actune.kernels.w4a8_triton as T4
    import actune.kernels.w8a8_triton as T8
    import actune.kernels.w2a8_triton as T2

    out = {}
    for w, mod, cls in ((4, T4, T4.W4A8TritonLinear), (8, T8, T8.W8A8TritonLinear), (2, T2, T2.W2A8TritonLinear)):
        for si, (m, k, n, with_bias) in enumerate(SHAPES):
            seed = 100 * w + si
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
            act = torch.empty(m, k, dtype=torch.int8)
            scale = torch.empty(m, dtype=torch.float32)
            T4._quantize_rows_kernel[(m,)](x, act, scale, in_features=k, BLOCK_K=256, num_warps=4)
            res = torch.empty(m, n, dtype=torch.float32)
            bias = layer.bias if layer.bias is not None else layer.weight_scale
            if w == 8:
                bm, bn, bk, nw = T8._config_for(m)
                T8._w8a8_gemm_kernel[(triton.cdiv(m, bm), triton.cdiv(n, bn))](
                    act, layer.weight_int8, scale, layer.weight_scale, bias, res, m, out_features=n, in_features=k,
                    has_bias=layer.bias is not None, BLOCK_M=bm, BLOCK_N=bn, BLOCK_K=bk, num_warps=nw)
                wbuf = layer.weight_int8.numpy()
                codes = layer.weight_int8.t().contiguous().numpy()
            elif w == 4:
                bm, bn, bj, nw = T4._config_for(m, n, k)
                T4._w4a8_gemm_kernel[(triton.cdiv(m, bm), triton.cdiv(n, bn))](
                    act, layer.packed_weight, scale, layer.weight_scale, bias, res, m, out_features=n,
                    in_features=k, has_bias=layer.bias is not None, BLOCK_M=bm, BLOCK_N=bn, BLOCK_J=bj,
                    num_warps=nw)
                wbuf = layer.packed_weight.numpy()
                p = layer.packed_weight.t().to(torch.int16)
                lo, hi = ((p & 15) ^ 8) - 8, (((p >> 4) & 15) ^ 8) - 8
                codes = torch.cat([lo, hi], 1).to(torch.int8).numpy()
            else:
                bm, bn, bj, nw = T2._config_for(m)
                T2._w2a8_gemm_kernel[(triton.cdiv(m, bm), triton.cdiv(n, bn))](
                    act, layer.packed_weight, scale, layer.weight_scale, bias, res, m, out_features=n,
                    in_features=k, has_bias=layer.bias is not None, BLOCK_M=bm, BLOCK_N=bn, BLOCK_J=bj,
                    num_warps=nw)
                wbuf = layer.packed_weight.numpy()
                p = layer.packed_weight.t().to(torch.int16)
                codes = torch.cat([(((p >> (2 * i)) & 3) ^ 2) - 2 for i in range(4)], 1).to(torch.int8).numpy()
            # Cross-check: the dot product of the codes is what the kernel computed.
            acc = act.numpy().astype(np.int64) @ codes.astype(np.int64).T
            ref = ((acc.astype(np.float32) * scale.numpy()[:, None]) * layer.weight_scale.numpy()[None, :])
            if layer.bias is not None:
                ref = ref + layer.bias.float().numpy()[None, :]
            assert np.abs(ref - res.numpy()).max() <= 1e-3 * max(1.0, np.abs(ref).max()), (w, si)
            key = f"w{w}_s{si}"
            out[f"{key}_x"] = x.view(torch.int16).numpy().view(np.uint16)
            out[f"{key}_weight"] = lin.weight.detach().view(torch.int16).numpy().view(np.uint16)
            out[f"{key}_act"] = act.numpy()
            out[f"{key}_scale"] = scale.numpy()
            out[f"{key}_codes"] = codes
            out[f"{key}_wbuf"] = wbuf
            out[f"{key}_ws"] = layer.weight_scale.numpy()
            if layer.bias is not None:
                out[f"{key}_bias"] = layer.bias.view(torch.int16).numpy().view(np.uint16)
            out[f"{key}_out"] = res.numpy()
            print(key, "ok", flush=True)
    np.savez_compressed(Path(args.out) / "tokenwise.npz", **out)
    print("tokenwise.npz", len(out))


if __name__ == "__main__":
    main()
