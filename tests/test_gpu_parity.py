"""GPU parity: the sm_100a kernels (through the C ABI) against the pinned CPU oracle.

Bar: bit-exact for everything integer (codes, scales, packed bytes, per-group
int32 dots) and, because the kernels evaluate the reference GPU kernels' fp32
chain in the same order (fma per group, then fma with ws and bias), bit-exact
fp32/bf16 outputs against the oracle in FMA mode.  Against the reference
interpreter goldens (separate multiply/add) the bf16 outputs must agree within
max-abs 1e-2 x output RMS (the project's stated tolerance).
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
PAIRS = [(w, a) for w in (2, 4, 8) for a in (2, 4, 8)]
SHAPES = [(1, 64, 32), (17, 256, 96), (64, 1024, 64)]
DEV = "cuda"


def bf16_bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def f32_of_bits(bits):
    return torch.from_numpy(O.bf16_bits_to_f32(bits).copy())


def assert_bits(actual, expected, what):
    actual = np.ascontiguousarray(actual)
    expected = np.ascontiguousarray(expected)
    assert actual.shape == expected.shape, f"{what}: shape {actual.shape} != {expected.shape}"
    ua = actual.reshape(-1).view(f"u{actual.dtype.itemsize}")
    ue = expected.reshape(-1).view(f"u{expected.dtype.itemsize}")
    diff = np.flatnonzero(ua != ue)
    assert diff.size == 0, f"{what}: {diff.size} of {actual.size} differ, first at {diff[:5]}"


@pytest.fixture(scope="module")
def ops():
    from actune_b200 import _lib, ops as o
    _lib.device_error(reset=True)
    yield o
    code, site = _lib.device_error()
    assert code == 0, f"device error word {code} (site {site})"


@pytest.fixture(scope="module")
def gemm_golden():
    return np.load(GOLDEN / "gemm.npz")


def inputs(m, k, seed, outliers=True, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g)
    if outliers:
        cols = torch.randperm(k, generator=torch.Generator().manual_seed(seed))[: max(1, k // 100)]
        x[:, cols] *= 20.0
    return x.to(dtype)


def weight(n, k, seed):
    g = torch.Generator().manual_seed(seed + 7)
    return (torch.randn(n, k, generator=g) * 0.02).bfloat16()


# --------------------------------------------------------------------------- quantizer
@pytest.mark.parametrize("a", [2, 4, 8])
@pytest.mark.parametrize("case", [0, 1, 2])
def test_quantizer_golden(ops, a, case):
    q = np.load(GOLDEN / "quantize.npz")
    x = q[f"a{a}_c{case}_x"]
    xt = torch.from_numpy(x.view(np.int16).copy()).view(torch.bfloat16) if x.dtype == np.uint16 else torch.from_numpy(x)
    packed, scales = ops.quantize_group64(xt.to(DEV), a)
    assert_bits(packed.cpu().numpy(), q[f"a{a}_c{case}_packed"], "packed")
    assert_bits(scales.cpu().numpy(), q[f"a{a}_c{case}_scales"], "scales")


@pytest.mark.parametrize("a", [2, 4, 8])
@pytest.mark.parametrize("m,k", [(1, 64), (3, 128), (600, 4096), (7, 11008), (129, 16384)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_quantizer_random(ops, a, m, k, dtype):
    x = inputs(m, k, seed=m * 31 + k + a, dtype=dtype)
    x[0, :64] = 0  # an all-zero group
    packed, scales = ops.quantize_group64(x.to(DEV), a)
    if dtype == torch.bfloat16:
        ref_p, ref_s = O.quantize_group64(bf16_bits(x), a)
    else:
        ref_p, ref_s = O.quantize_group64(x.float().numpy(), a)
    assert_bits(packed.cpu().numpy(), ref_p, "packed")
    assert_bits(scales.cpu().numpy(), ref_s, "scales")


def test_quantizer_empty(ops):
    x = torch.empty(0, 128, device=DEV, dtype=torch.bfloat16)
    packed, scales = ops.quantize_group64(x, 8)
    assert packed.shape == (0, 128) and scales.shape == (0, 2)


# --------------------------------------------------------------------------- weight codes
@pytest.mark.parametrize("w,a", PAIRS)
@pytest.mark.parametrize("tag", ["noclip", "clip"])
def test_weight_codes_golden(ops, w, a, tag):
    d = np.load(GOLDEN / "weights.npz")
    wt = torch.from_numpy(d["weight"].view(np.int16).copy()).view(torch.bfloat16).to(DEV)
    clip = torch.from_numpy(d["clips"]).to(DEV) if tag == "clip" else None
    from actune_b200.kernels.quantizers import weight_codes
    codes, scale = weight_codes(wt, w, a, clip_ratios=clip)
    assert_bits(codes.cpu().numpy(), d[f"w{w}a{a}_{tag}_codes"], "codes")
    assert_bits(scale.cpu().numpy(), d[f"w{w}a{a}_{tag}_scale"], "scale")
    packed = ops.pack_rows(codes, w)
    assert_bits(packed.cpu().numpy(), d[f"w{w}a{a}_{tag}_packed"], "packed")


def test_signed_r4_refine_matches_nested_codes(ops):
    from actune_b200.kernels.quantizers import signed_r4_refine, symmetric_int4_quantize, weight_codes
    wt = weight(64, 256, 3).to(DEV)
    q4, s4 = symmetric_int4_quantize(wt)
    residual, q8 = signed_r4_refine(wt, q4, s4)
    nested, s8 = weight_codes(wt, 8, 4)
    assert torch.equal(q8, nested) and torch.equal(s8 * 16, s4)
    assert torch.equal(q8.to(torch.int16), 16 * q4.to(torch.int16) + residual.to(torch.int16))


# --------------------------------------------------------------------------- GEMM vs goldens
@pytest.mark.parametrize("w,a", PAIRS)
@pytest.mark.parametrize("si", [0, 1, 2])
def test_gemm_golden(ops, gemm_golden, w, a, si):
    m, k, n = SHAPES[si]
    key = f"s{si}_w{w}a{a}"
    g = gemm_golden
    pa = torch.from_numpy(g[f"{key}_pa"]).to(DEV)
    as_ = torch.from_numpy(g[f"{key}_as"]).to(DEV)
    pw = torch.from_numpy(g[f"{key}_pw"]).to(DEV)
    ws = torch.from_numpy(g[f"{key}_ws"]).to(DEV)
    bias = f32_of_bits(g[f"s{si}_bias"]).to(DEV)
    # AUTO, BN32/64/128, the weights-in-TMEM WT16/32/64/128 and (M <= 32) the
    # weight-streaming kernel.
    for variant in range(9 if m <= 32 else 8):
        dots = ops.packed_linear_dots(pa, pw, k, w, a, variant=variant).cpu().numpy()
        ref = g[f"{key}_dots"]
        assert np.array_equal(dots[: ref.shape[0]], ref), f"dots variant {variant}"
        y32 = ops.packed_linear(pa, as_, pw, ws, bias, k, w, a, out_dtype=torch.float32, variant=variant)
        exact = O.packed_linear(g[f"{key}_pa"], g[f"{key}_as"], g[f"{key}_pw"], g[f"{key}_ws"],
                                O.bf16_bits_to_f32(g[f"s{si}_bias"]), k, w, a, fma=True)
        assert_bits(y32.cpu().numpy(), exact, f"fp32 output variant {variant}")
        # Against the reference run under the Triton interpreter (separate
        # multiply and add, no FMA), both rounded to bf16: the two evaluation
        # modes of the reference itself may differ by one bf16 ulp where the
        # fp32 values straddle a rounding boundary; nothing else may differ.
        ref_bits = O.to_bf16_bits(g[f"{key}_y"])
        yb = ops.packed_linear(pa, as_, pw, ws, bias, k, w, a, out_dtype=torch.bfloat16, variant=variant)
        ours = bf16_bits(yb).astype(np.int32)
        ulps = np.abs(ours - ref_bits.astype(np.int32))
        assert ulps.max() <= 1 and (ulps > 0).mean() <= 0.01, f"{(ulps > 0).sum()} elements differ"


# --------------------------------------------------------------------------- GEMM random / edge shapes
def _case(ops, m, k, n, w, a, seed, bias_dtype=torch.bfloat16, out_dtype=torch.bfloat16, variant=0, rows=None):
    x = inputs(m, k, seed)
    wt = weight(n, k, seed)
    codes, ws = ops.weight_codes(wt.to(DEV), w, a)
    pw = ops.pack_rows(codes, w)
    pa, as_ = ops.quantize_group64(x.to(DEV), a)
    bias = None if bias_dtype is None else (torch.randn(n, generator=torch.Generator().manual_seed(seed)) * 0.1).to(
        bias_dtype)
    y = ops.packed_linear(pa, as_, pw, ws, None if bias is None else bias.to(DEV), k, w, a, out_dtype=out_dtype,
                          variant=variant)
    sel = np.arange(m) if rows is None else np.asarray(rows)
    pa_h, as_h = pa.cpu().numpy()[sel], as_.cpu().numpy()[sel]
    ref = O.packed_linear(pa_h, as_h, pw.cpu().numpy(), ws.cpu().numpy(),
                          None if bias is None else bias.float().numpy(), k, w, a, fma=True)
    return y.cpu()[torch.from_numpy(sel)], ref, (pa, pw, pa_h)


@pytest.mark.parametrize("w,a", PAIRS)
@pytest.mark.parametrize("m,k,n", [(1, 4096, 4096), (8, 4096, 12288), (130, 1024, 200), (300, 192, 136)])
def test_gemm_random_bit_exact(ops, w, a, m, k, n):
    y, ref, _ = _case(ops, m, k, n, w, a, seed=m + k + n + 10 * w + a)
    assert_bits(bf16_bits(y), O.to_bf16_bits(ref), "bf16 output")


@pytest.mark.parametrize("w", [2, 4, 8])
@pytest.mark.parametrize("m", [1, 20, 33, 50, 57, 64])
def test_gemm_single_token_tile(ops, w, m):
    """One tile of at most 64 int8 token rows (a token box only as high as the tokens;
    every tile width, the wave-tail split included): fp32 and bf16 outputs bit-exact
    against the oracle, with and without bias, odd and even group counts, ragged N."""
    for k, n, bias_dtype in [(448, 200, torch.bfloat16), (1024, 1000, None), (128, 12288, torch.float32),
                             (256, 20480, None)]:
        for variant in (0, 1, 2, 3):
            seed = m + k + n + 10 * w + variant
            y, ref, _ = _case(ops, m, k, n, w, 8, seed, bias_dtype=bias_dtype, out_dtype=torch.float32,
                              variant=variant)
            assert_bits(y.numpy(), ref, f"fp32 m={m} k={k} n={n} variant={variant}")
    y, ref, _ = _case(ops, m, 4096, 2560, w, 8, seed=m + w, variant=1)
    assert_bits(bf16_bits(y), O.to_bf16_bits(ref), f"bf16 output m={m} 4096x2560 BN32")


@pytest.mark.parametrize("w,a", PAIRS)
@pytest.mark.parametrize("variant", [9, 10, 11])
def test_gemm_two_ctas_per_sm_variants(ops, w, a, variant):
    """BN32X2 / BN64X2 / BN128X2 (two CTAs per SM, half the tensor memory each, one
    accumulator pair at BN=128) on ragged shapes and a multi-wave one: bit-exact, and
    the debug dots export through them runs the one-CTA kernel."""
    for m, k, n in [(37, 448, 200), (300, 1024, 1000)]:
        y, ref, (pa, pw, pa_h) = _case(ops, m, k, n, w, a, seed=m + k + n + variant, variant=variant)
        assert_bits(bf16_bits(y), O.to_bf16_bits(ref), f"bf16 output m={m} k={k} n={n}")
    d = ops.packed_linear_dots(pa, pw, k, w, a, variant=variant)
    assert torch.equal(d, ops.packed_linear_dots(pa, pw, k, w, a, variant=3))


@pytest.mark.parametrize("w,a", [(4, 8), (8, 8), (2, 2), (4, 4)])
@pytest.mark.parametrize("m,k,n", [(600, 256, 12288), (600, 192, 3990), (600, 128, 4096)])
def test_gemm_auto_split_waves(ops, w, a, m, k, n):
    """AUTO splits a GEMM whose 128-column tiles leave a partial last wave into a
    launch for the whole waves and a second, programmatically dependent launch of
    narrower tiles for the remaining columns (BN=64 for the first shape, BN=32 for the
    others, a ragged tail for N=3990): identical to the unsplit kernel, and sampled
    rows bit-exact against the oracle."""
    rows = [0, 127, 128, 599]
    y, ref, (pa, pw, pa_h) = _case(ops, m, k, n, w, a, seed=m + k + n + w, out_dtype=torch.float32, rows=rows)
    assert_bits(y.numpy(), ref, f"fp32 output m={m} k={k} n={n}")
    x = inputs(m, k, m + k + n + w).to(DEV)
    wt = weight(n, k, m + k + n + w).to(DEV)
    codes, ws = ops.weight_codes(wt, w, a)
    pw = ops.pack_rows(codes, w)
    pa, as_ = ops.quantize_group64(x, a)
    auto = ops.packed_linear(pa, as_, pw, ws, None, k, w, a, out_dtype=torch.bfloat16, variant=0)
    whole = ops.packed_linear(pa, as_, pw, ws, None, k, w, a, out_dtype=torch.bfloat16, variant=3)
    assert torch.equal(auto, whole)


@pytest.mark.parametrize("m", [33, 50, 64, 100, 128, 200, 304])
@pytest.mark.parametrize("k,n", [(64, 200), (192, 1000), (1088, 1024), (4096, 2560), (1024, 8192)])
def test_gemm_four_group_stages(ops, m, k, n):
    """AUTO on int8 codes (W = A = 8, the decoded path every pair takes above 32 token
    rows) with a 32- or 64-column tile runs the four-group-stage kernel: one to three
    token tiles, 1, 3, 17, 64 and 16 groups (partial and whole last stages), ragged N,
    with and without bias, three output types -- bit-exact against the oracle and
    identical to the two-group-stage kernel (explicit BN32 and BN64)."""
    for bias_dtype, out_dtype in [(torch.bfloat16, torch.bfloat16), (None, torch.float32),
                                  (torch.float32, torch.float16)]:
        seed = m + k + n + (0 if bias_dtype is None else 1)
        y, ref, (pa, pw, pa_h) = _case(ops, m, k, n, 8, 8, seed, bias_dtype=bias_dtype, out_dtype=out_dtype)
        if out_dtype == torch.float32:
            assert_bits(y.numpy(), ref, f"fp32 m={m} k={k} n={n}")
        elif out_dtype == torch.bfloat16:
            assert_bits(bf16_bits(y), O.to_bf16_bits(ref), f"bf16 m={m} k={k} n={n}")
        for variant in (1, 2):
            y2, _, _ = _case(ops, m, k, n, 8, 8, seed, bias_dtype=bias_dtype, out_dtype=out_dtype, variant=variant)
            assert torch.equal(y.view(torch.int16) if y.dtype != torch.float32 else y.view(torch.int32),
                               y2.view(torch.int16) if y2.dtype != torch.float32 else y2.view(torch.int32)), \
                f"AUTO vs variant {variant} m={m} k={k} n={n} {out_dtype}"


@pytest.mark.parametrize("w,a", [p for p in PAIRS if p != (8, 8)])
@pytest.mark.parametrize("m", [50, 200])
@pytest.mark.parametrize("k,n", [(192, 1000), (1088, 264), (1024, 2560)])
def test_gemm_four_group_stages_packed(ops, w, a, m, k, n):
    """AUTO on packed sub-byte codes with a 32- or 64-column tile: the four-group-stage
    kernel with its converter warps (packed codes expanded to int8 in shared memory)
    where its ring holds four stages (W2A2, W2A8, W4A8, W8A2 at 32 columns), the
    two-group-stage kernel otherwise -- bit-exact against the oracle and identical to
    the explicit BN32 / BN64 variants, odd and even group counts, one and two token
    tiles."""
    seed = m + k + n + 10 * w + a
    y, ref, _ = _case(ops, m, k, n, w, a, seed, out_dtype=torch.float32)
    assert_bits(y.numpy(), ref, f"fp32 W{w}A{a} m={m} k={k} n={n}")
    for variant in (1, 2):
        y2, _, _ = _case(ops, m, k, n, w, a, seed, out_dtype=torch.float32, variant=variant)
        assert torch.equal(y.view(torch.int32), y2.view(torch.int32)), f"AUTO vs variant {variant}"


@pytest.mark.parametrize("w,a", [(8, 8), (4, 8), (8, 4), (2, 2)])
@pytest.mark.parametrize("m,k,n", [(300, 192, 136), (260, 1024, 256), (50, 192, 136), (100, 1088, 2560)])
def test_gemm_extreme_codes_and_scales(ops, w, a, m, k, n):
    """Raw codes at both ends of their range (|dot| up to 2^20, the largest an int8
    group dot reaches), activation scales near 2^105 (products near 2^125), subnormal
    and zero scales, an odd group count and a ragged N, over several token tiles:
    fp32 and bf16 outputs bit-exact against the oracle for tile widths 128 and 64 and
    AUTO."""
    g = torch.Generator().manual_seed(m + k + n + 10 * w + a)
    lo_a, hi_a = -(1 << (a - 1)), (1 << (a - 1)) - 1
    lo_w, hi_w = -(1 << (w - 1)), (1 << (w - 1)) - 1
    qa = torch.randint(lo_a, hi_a + 1, (m, k), generator=g, dtype=torch.int8)
    qw = torch.randint(lo_w, hi_w + 1, (n, k), generator=g, dtype=torch.int8)
    qa[0], qa[1], qa[2] = lo_a, hi_a, lo_a
    qa[2, 1::2] = hi_a
    qw[0], qw[1] = lo_w, hi_w
    G = k // 64
    as_ = torch.empty(m, G).uniform_(1e-3, 1e-1, generator=g)
    as_[3, 0] = 2.0 ** 105                  # s * 2^23 overflows: conversion path
    as_[4, 0] = 2.0 ** 104 * 1.9990234375   # largest kind of scale still carried
    as_[5, :] = 2.0 ** 105                  # every group (odd ones keep the hardware conversion)
    as_[5, 1:] = 1e-3
    as_[6, :] = 1e-40                       # subnormal
    as_[7, 0] = 0.0
    as_[0, 0] = 2.0 ** 105                  # with the largest dot
    ws = torch.empty(n).uniform_(1e-3, 2e-2, generator=g)
    bias = torch.randn(n, generator=g) * 0.1
    pa = ops.pack_rows(qa.to(DEV), a)
    pw = ops.pack_rows(qw.to(DEV), w)
    ref = O.packed_linear(pa.cpu().numpy(), as_.numpy(), pw.cpu().numpy(), ws.numpy(), bias.numpy(), k, w, a,
                          fma=True)
    assert np.isfinite(ref).all()
    for variant in (3, 2, 0):  # BN128 (preset), BN64 (plain), AUTO
        y = ops.packed_linear(pa, as_.to(DEV), pw, ws.to(DEV), bias.to(DEV), k, w, a, out_dtype=torch.float32,
                              variant=variant)
        assert_bits(y.cpu().numpy(), ref, f"fp32 variant {variant}")
        yb = ops.packed_linear(pa, as_.to(DEV), pw, ws.to(DEV), bias.to(DEV), k, w, a, out_dtype=torch.bfloat16,
                               variant=variant)
        assert_bits(bf16_bits(yb), O.to_bf16_bits(ref), f"bf16 variant {variant}")


@pytest.mark.parametrize("w,a", PAIRS)
@pytest.mark.parametrize("variant", [12, 13])
def test_gemm_persistent_variants(ops, w, a, variant):
    """BN64P / BN128P (one CTA per SM walking the tiles, TMA-store epilogue): ragged
    tiles, an odd number of K groups, more tiles than SMs (each CTA takes several),
    bf16 and f16 outputs bit-exact; fp32 outputs and N % 8 != 0 fall back to the
    one-tile kernel."""
    for m, k, n, out_dtype in [(37, 448, 200, torch.bfloat16), (300, 1024, 1000, torch.float16),
                               (600, 2048, 4096, torch.bfloat16), (129, 192, 136, torch.float32),
                               (70, 256, 100, torch.bfloat16)]:
        y, ref, _ = _case(ops, m, k, n, w, a, seed=m + k + n + variant, out_dtype=out_dtype, variant=variant)
        if out_dtype == torch.float32:
            assert_bits(y.numpy(), ref, f"fp32 output m={m} k={k} n={n}")
        elif out_dtype == torch.float16:
            assert_bits(y.view(torch.int16).numpy().view(np.uint16), ref.astype(np.float16).view(np.uint16),
                        f"f16 output m={m} k={k} n={n}")
        else:
            assert_bits(bf16_bits(y), O.to_bf16_bits(ref), f"bf16 output m={m} k={k} n={n}")


@pytest.mark.parametrize("w,a", PAIRS)
@pytest.mark.parametrize("variant", [4, 5, 6, 7])
def test_gemm_weights_in_tmem_variants(ops, w, a, variant):
    """The weights-in-TMEM kernel (explicit WT variants) on ragged shapes: partial
    weight tiles, partial token tiles and an odd number of K groups."""
    for m, k, n in [(37, 448, 200), (130, 1024, 136)]:
        y, ref, _ = _case(ops, m, k, n, w, a, seed=m + k + n + variant, variant=variant)
        assert_bits(bf16_bits(y), O.to_bf16_bits(ref), f"bf16 output m={m} k={k} n={n}")


DECODE_SHAPES = [
    (1, 1536, 200),   # whole-stage boxes, partial last stage, ragged N
    (5, 3072, 4800),  # whole-stage boxes, more 32-row blocks than SMs (persistent loop)
    (16, 512, 96),    # whole-stage boxes, half a stage: K-lanes 2 and 3 see only padding
    (3, 448, 72),     # packed rows not a multiple of 128 bytes: one 2-D box per block, 2048-K stage
    (9, 1088, 200),   # 2-D boxes, 16-token tile, partial last block of every row
    (4, 2240, 64),    # 2-D boxes, 2048-K stages (the second one partial)
    (1, 11008, 136),  # the Llama down-projection K: 2-bit rows are 2,752 bytes
    (24, 4096, 136),  # 17..32 tokens
    (32, 1024, 64),
]


@pytest.mark.parametrize("w,a", PAIRS)
@pytest.mark.parametrize("m,k,n", DECODE_SHAPES)
def test_gemm_weight_streaming_variant(ops, w, a, m, k, n):
    """The weight-streaming kernels (VARIANT_GEMV, and AUTO at M <= 32): fp32 output
    bit-exact, per-group dots equal to the oracle's."""
    y, ref, (pa, pw, pa_h) = _case(ops, m, k, n, w, a, seed=m + k + n + w * a, out_dtype=torch.float32,
                                   variant=8)
    assert_bits(y.numpy(), ref, f"fp32 output m={m} k={k} n={n}")
    dots = ops.packed_linear_dots(pa, pw, k, w, a, variant=8).cpu().numpy()
    assert np.array_equal(dots, O.group_dots(pa_h, pw.cpu().numpy(), k, w, a))
    assert torch.equal(ops.packed_linear_dots(pa, pw, k, w, a, variant=0).cpu(), torch.from_numpy(dots))


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("bias_dtype", [None, torch.float32, torch.float16, torch.bfloat16])
def test_gemm_dtypes(ops, out_dtype, bias_dtype):
    y, ref, _ = _case(ops, 70, 384, 100, 4, 8, seed=5, bias_dtype=bias_dtype, out_dtype=out_dtype)
    if out_dtype == torch.float32:
        assert_bits(y.numpy(), ref, "fp32 output")
    elif out_dtype == torch.bfloat16:
        assert_bits(bf16_bits(y), O.to_bf16_bits(ref), "bf16 output")
    else:
        assert torch.equal(y, torch.from_numpy(ref).half())


@pytest.mark.parametrize("w,a", [(4, 8), (4, 4), (2, 2), (8, 8)])
def test_gemm_llama_shapes_row_sample(ops, w, a):
    """Config-1 shapes at M=512: 8 sampled rows against the oracle (rows are independent)."""
    rows = [0, 1, 127, 128, 255, 300, 510, 511]
    for k, n in [(4096, 12288), (4096, 4096), (4096, 22016), (11008, 4096)]:
        y, ref, _ = _case(ops, 512, k, n, w, a, seed=k + n, rows=rows)
        assert_bits(bf16_bits(y), O.to_bf16_bits(ref), f"bf16 output K={k} N={n}")


def test_gemm_dots_full_size_properties(ops):
    """Full-size W4A8 QKV: the per-group dots equal the oracle on sampled rows and
    are invariant to the tile variant."""
    m, k, n, w, a = 600, 4096, 12288, 4, 8
    x = inputs(m, k, 11)
    codes, ws = ops.weight_codes(weight(n, k, 11).to(DEV), w, a)
    pw = ops.pack_rows(codes, w)
    pa, as_ = ops.quantize_group64(x.to(DEV), a)
    d0 = ops.packed_linear_dots(pa, pw, k, w, a, variant=3)
    d1 = ops.packed_linear_dots(pa, pw, k, w, a, variant=1)
    assert torch.equal(d0, d1)
    assert torch.equal(d0, ops.packed_linear_dots(pa, pw, k, w, a, variant=7))
    rows = [0, 99, 511, 599]
    ref = O.group_dots(pa.cpu().numpy()[rows], pw.cpu().numpy(), k, w, a)
    assert np.array_equal(d0.cpu().numpy()[rows], ref)


def test_gemm_empty(ops):
    pa = torch.empty(0, 64, device=DEV, dtype=torch.uint8)
    as_ = torch.empty(0, 1, device=DEV, dtype=torch.float32)
    pw = torch.zeros(32, 32, device=DEV, dtype=torch.uint8)
    ws = torch.ones(32, device=DEV)
    y = ops.packed_linear(pa, as_, pw, ws, None, 64, 4, 8)
    assert y.shape == (0, 32)


def test_gemm_rejects_bad_arguments(ops):
    from actune_b200._lib import ActuneError
    pa = torch.zeros(4, 64, device=DEV, dtype=torch.uint8)
    as_ = torch.ones(4, 1, device=DEV)
    pw = torch.zeros(32, 32, device=DEV, dtype=torch.uint8)
    ws = torch.ones(32, device=DEV)
    with pytest.raises(RuntimeError):
        ops.packed_linear(pa, as_, pw, ws, None, 64, 3, 8)      # W outside {2,4,8}
    with pytest.raises(RuntimeError):
        ops.packed_linear(pa, as_, pw, ws, None, 63, 4, 8)      # K not a multiple of 64
    shifted = torch.zeros(4 * 64 + 1, device=DEV, dtype=torch.uint8)[1:].view(4, 64)
    with pytest.raises(ActuneError) as err:
        ops.packed_linear(shifted, as_, pw, ws, None, 64, 4, 8)  # TMA needs 16-byte alignment
    assert err.value.status == 2
