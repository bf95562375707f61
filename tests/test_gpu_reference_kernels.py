"""The reference's own CUDA kernels, run on the B200, as a GPU-side checker.

oracle/build_ref.py compiles the reference's native extensions from its sources
(actune/kernels/grouped_native.cu, grouped_big_m.cu, native_s4_extension.cpp +
native_s4_extension_kernel.cu) for sm_100a with the reference's own flags into
oracle/_ref/.  Where those modules were built, these tests feed them and this
library the same packed operands and require bit-identical outputs:

* group-64 W{2,4} x A{2,4} (``linear(a, as, w, ws, bias, source, W, A)`` and its 13
  tuned geometries): pins the fp32 chain order -- fma(float(dot), as, acc) per
  group, then fma(acc, ws, bias) -- by executing the reference's kernel, not only
  by reading it;
* per-row A4 W{2,4}A4 (``linear(packed_activation, activation_scale,
  packed_weight, weight_scale, bias, output_template, weight_bits)``): pins the
  native epilogue float(acc) * (as * ws) (+ bias) the same way.

When a module is absent (the reference was not mounted where the library was
built) the test is skipped and says so.
"""
import numpy as np
import pytest
import torch

from oracle import build_ref

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _module(name):
    mod = build_ref.load(name)
    if mod is None:
        pytest.skip(f"{name} not built (oracle/build_ref.py needs the reference sources)")
    return mod


def bf16_bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.fixture(scope="module")
def ops():
    from actune_b200 import _lib, ops as o
    _lib.device_error(reset=True)
    yield o
    code, site = _lib.device_error()
    assert code == 0, f"device error word {code} (site {site})"


def _operands(ops, m, k, n, w, a, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g)
    x[:, torch.randperm(k, generator=g)[: max(1, k // 100)]] *= 20.0
    x = x.bfloat16().to(DEV)
    wt = (torch.randn(n, k, generator=g) * 0.02).bfloat16().to(DEV)
    codes, ws = ops.weight_codes(wt, w, a)
    pw = ops.pack_rows(codes, w)
    pa, as_ = ops.quantize_group64(x, a)
    bias = (torch.randn(n, generator=g) * 0.1).float().to(DEV)
    return x, pa, as_, pw, ws, bias


@pytest.mark.parametrize("w,a", [(2, 2), (2, 4), (4, 2), (4, 4)])
@pytest.mark.parametrize("m,k,n", [(1, 256, 64), (37, 1024, 200), (600, 4096, 512)])
def test_reference_group64_kernel_matches(ops, w, a, m, k, n):
    ref = _module("ref_grouped_native")
    x, pa, as_, pw, ws, bias = _operands(ops, m, k, n, w, a, seed=m + k + n + w + a)
    for b in (bias, torch.empty(0, device=DEV)):
        want = ref.linear(pa, as_, pw, ws, b, x, w, a)
        ours = ops.packed_linear(pa, as_, pw, ws, b if b.numel() else None, k, w, a, out_dtype=torch.bfloat16)
        assert np.array_equal(bf16_bits(ours), bf16_bits(want)), \
            f"{int((bf16_bits(ours) != bf16_bits(want)).sum())} of {ours.numel()} differ (bias={b.numel() > 0})"
        want32 = ref.linear(pa, as_, pw, ws, b, x.float(), w, a)
        ours32 = ops.packed_linear(pa, as_, pw, ws, b if b.numel() else None, k, w, a, out_dtype=torch.float32)
        assert torch.equal(ours32, want32)


@pytest.mark.parametrize("w,a", [(4, 4), (2, 4)])
def test_reference_tuned_geometries_match(ops, w, a):
    ref = _module("ref_grouped_big_m")
    m, k, n = 300, 2048, 384
    x, pa, as_, pw, ws, bias = _operands(ops, m, k, n, w, a, seed=77)
    ours = bf16_bits(ops.packed_linear(pa, as_, pw, ws, bias, k, w, a, out_dtype=torch.bfloat16))
    for config in range(13):
        want = bf16_bits(ref.linear(pa, as_, pw, ws, bias, x, w, a, config))
        assert np.array_equal(ours, want), f"config {config}"


@pytest.mark.parametrize("wbits", [2, 4])
@pytest.mark.parametrize("m,k,n", [(5, 512, 96), (200, 4096, 384)])
def test_reference_native_s4_epilogue_matches(wbits, m, k, n):
    ref = _module("ref_native_s4")
    from actune_b200.kernels.wxa4_native import W2A4NativeLinear, W4A4NativeLinear
    g = torch.Generator().manual_seed(m + k + wbits)
    linear = torch.nn.Linear(k, n, bias=True, dtype=torch.bfloat16)
    with torch.no_grad():
        linear.weight.copy_((torch.randn(n, k, generator=g) * 0.02).bfloat16())
        linear.bias.copy_((torch.randn(n, generator=g) * 0.1).bfloat16())
    linear = linear.to(DEV)
    module = (W2A4NativeLinear if wbits == 2 else W4A4NativeLinear)(linear)
    x = torch.randn(m, k, generator=g).bfloat16().to(DEV)
    ours = module(x)
    from actune_b200 import ops
    pa, as_ = ops.quantize_rows_a4(x)
    want = ref.linear(pa, as_, module.packed_weight, module.weight_scale, module.bias, x, wbits)
    diff = int((bf16_bits(ours) != bf16_bits(want)).sum())
    assert diff == 0, f"{diff} of {ours.numel()} differ"
