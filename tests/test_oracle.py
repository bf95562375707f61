"""The CPU oracle against the golden vectors produced by the reference's own code.

This pins the oracle: if it passes, oracle/group64.c reproduces the reference's
activation quantizer (actune/kernels/grouped.py:55-71), weight codebooks
(actune/kernels/quantizers.py:23-94), packing (grouped.py:108-111), per-group
int32 dots and fp32 epilogue (grouped.py:74-94) bit for bit.
"""
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"
PAIRS = [(w, a) for w in (2, 4, 8) for a in (2, 4, 8)]
SHAPES = [(1, 64, 32), (17, 256, 96), (64, 1024, 64)]


@pytest.fixture(scope="module")
def quant():
    return np.load(GOLDEN / "quantize.npz")


@pytest.fixture(scope="module")
def weights():
    return np.load(GOLDEN / "weights.npz")


@pytest.fixture(scope="module")
def gemm():
    return np.load(GOLDEN / "gemm.npz")


def bits_equal(a, b):
    a, b = np.asarray(a), np.asarray(b)
    return a.shape == b.shape and np.array_equal(a.view(np.uint8), b.view(np.uint8))


@pytest.mark.parametrize("a", [2, 4, 8])
@pytest.mark.parametrize("case", [0, 1, 2])
def test_quantizer_matches_reference(quant, a, case):
    x = quant[f"a{a}_c{case}_x"]
    packed, scales = O.quantize_group64(x, a)
    assert bits_equal(packed, quant[f"a{a}_c{case}_packed"])
    assert bits_equal(scales, quant[f"a{a}_c{case}_scales"])


@pytest.mark.parametrize("w,a", PAIRS)
@pytest.mark.parametrize("tag", ["noclip", "clip"])
def test_weight_codes_match_reference(weights, w, a, tag):
    wf = O.bf16_bits_to_f32(weights["weight"])
    clip = weights["clips"] if tag == "clip" else None
    codes, scale = O.weight_codes(wf, w, a, clip)
    assert bits_equal(codes, weights[f"w{w}a{a}_{tag}_codes"])
    assert bits_equal(scale, weights[f"w{w}a{a}_{tag}_scale"])
    packed = O.pack_rows(codes, w)
    assert bits_equal(packed, weights[f"w{w}a{a}_{tag}_packed"])
    assert bits_equal(O.unpack_rows(packed, wf.shape[1], w), codes)


@pytest.mark.parametrize("w,a", PAIRS)
@pytest.mark.parametrize("si", [0, 1, 2])
def test_gemm_matches_reference(gemm, w, a, si):
    m, k, n = SHAPES[si]
    key = f"s{si}_w{w}a{a}"
    x = gemm[f"s{si}_x"]
    pa, as_ = O.quantize_group64(x, a)
    assert bits_equal(pa, gemm[f"{key}_pa"]) and bits_equal(as_, gemm[f"{key}_as"])
    wf = O.bf16_bits_to_f32(gemm[f"s{si}_weight"])
    codes, ws = O.weight_codes(wf, w, a)
    pw = O.pack_rows(codes, w)
    assert bits_equal(pw, gemm[f"{key}_pw"]) and bits_equal(ws, gemm[f"{key}_ws"])
    dots = O.group_dots(pa, pw, k, w, a)
    ref_dots = gemm[f"{key}_dots"]
    assert np.array_equal(dots[: ref_dots.shape[0]], ref_dots)
    bias = O.bf16_bits_to_f32(gemm[f"s{si}_bias"])
    # Interpreter arithmetic = separate multiply and add.
    y = O.packed_linear(pa, as_, pw, ws, bias, k, w, a, fma=False)
    assert bits_equal(y, gemm[f"{key}_y"])
    if si == 1:
        y0 = O.packed_linear(pa, as_, pw, ws, None, k, w, a, fma=False)
        assert bits_equal(y0, gemm[f"{key}_y_nobias"])
    # The fused (GPU-reference) mode stays within fp32 rounding of the unfused one.
    yf = O.packed_linear(pa, as_, pw, ws, bias, k, w, a, fma=True)
    rms = float(np.sqrt(np.mean(y.astype(np.float64) ** 2))) + 1e-30
    assert float(np.max(np.abs(yf - y))) <= 1e-5 * rms * max(1, k // 64)


def test_bf16_rounding_is_rne():
    vals = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.4e38, 1e-40], np.float32)
    bits = O.to_bf16_bits(vals)
    import torch
    ref = torch.from_numpy(vals).bfloat16().view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(bits, ref)


# ---------------------------------------------------------------------------- tokenwise backends
@pytest.fixture(scope="module")
def tokenwise():
    return np.load(GOLDEN / "tokenwise.npz")


@pytest.mark.parametrize("w", [4, 8, 2])
@pytest.mark.parametrize("si", [0, 1, 2])
def test_tokenwise_matches_reference(tokenwise, w, si):
    """Per-row A8 quantizer (reciprocal-multiply scale), the W{4,8,2} codebooks and
    the full-K int32 GEMM with its fp32 epilogue, against the reference's
    W{4,8,2}A8TritonLinear kernels run under the Triton interpreter."""
    g, key = tokenwise, f"w{w}_s{si}"
    codes_a, scale = O.quantize_rows_a8(g[f"{key}_x"])
    assert bits_equal(codes_a, g[f"{key}_act"]) and bits_equal(scale, g[f"{key}_scale"])
    wq, ws = O.weight_codes(O.bf16_bits_to_f32(g[f"{key}_weight"]), w, 8)
    assert bits_equal(wq, g[f"{key}_codes"]) and bits_equal(ws, g[f"{key}_ws"])
    bias = O.bf16_bits_to_f32(g[f"{key}_bias"]) if f"{key}_bias" in g else None
    y = O.tokenwise_linear(codes_a, scale, wq, ws, bias, fma=False)  # interpreter: separate multiply and add
    assert bits_equal(y, g[f"{key}_out"])
    yf = O.tokenwise_linear(codes_a, scale, wq, ws, bias, fma=True)
    assert float(np.max(np.abs(yf - y))) <= 1e-6 * (float(np.abs(y).max()) + 1e-30)


@pytest.fixture(scope="module")
def wxa4():
    return np.load(GOLDEN / "wxa4.npz")


@pytest.mark.parametrize("w", [2, 4, 8])
@pytest.mark.parametrize("si", [0, 1, 2])
def test_wxa4_matches_reference(wxa4, w, si):
    """Per-row A4 quantizer (packed nibbles, reciprocal-multiply scale) and its INT8
    sign extension, the W{2,4} codebooks and the nested W8 code of W8A4, and the
    W8A4 GEMM (the W8A8 Triton kernel on sign-extended A4 codes), against the
    reference's W{2,4,8}A4NativeLinear run under the Triton interpreter."""
    g, key = wxa4, f"w{w}_s{si}"
    packed, scale = O.quantize_rows_a4(g[f"{key}_x"])
    assert bits_equal(packed, g[f"{key}_packed"]) and bits_equal(scale, g[f"{key}_scale"])
    act = O.unpack_a4(packed)
    assert bits_equal(act, g[f"{key}_act"])
    wq, ws = O.weight_codes(O.bf16_bits_to_f32(g[f"{key}_weight"]), w, 4)
    assert bits_equal(wq, g[f"{key}_codes"]) and bits_equal(ws, g[f"{key}_ws"])
    bias = g[f"{key}_bias"] if f"{key}_bias" in g else None
    if w == 8:
        y = O.tokenwise_linear(act, scale, wq, ws, bias, fma=False)  # interpreter: separate multiply and add
        assert bits_equal(y, g[f"{key}_out"])
    else:
        # The native kernel's epilogue: float(acc) * (as * ws) (+ bias); against the
        # exact product in float64 it stays within a few fp32 roundings.
        y = O.rowwise_native_linear(act, scale, wq, ws, bias, fma=True)
        acc = act.astype(np.int64) @ wq.astype(np.int64).T
        ref = acc.astype(np.float64) * scale.astype(np.float64)[:, None] * ws.astype(np.float64)[None, :]
        if bias is not None:
            ref = ref + bias.astype(np.float64)[None, :]
        assert np.abs(y - ref).max() <= 4e-7 * max(1.0, np.abs(ref).max())
