"""Per-row A4 backends (W2A4 / W4A4 / W8A4) on the GPU against the oracle and the
reference's goldens.

The goldens (tests/golden/wxa4.npz, made by tests/golden/gen_wxa4.py) hold the
reference's A4 quantizer output, module buffers and, for W8A4, the output of the
W8A8 Triton kernel it runs (fp32, separate multiply and add); the oracle reproduces
them bit for bit (tests/test_oracle.py).  The GPU epilogues fuse the last multiply
and add as the reference's GPU kernels do, so fp32 outputs are compared with the
oracle's FMA mode bit for bit.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
DEV = "cuda"


@pytest.fixture(scope="module")
def g():
    return np.load(GOLDEN / "wxa4.npz")


@pytest.fixture(scope="module")
def ops():
    from actune_b200 import ops as o
    return o


@pytest.fixture(autouse=True)
def device_error_word_clean():
    from actune_b200 import _lib
    _lib.device_error(reset=True)
    yield
    assert _lib.device_error()[0] == 0


def bf16_tensor(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


def bits_equal(a, b):
    a, b = np.asarray(a), np.asarray(b)
    return a.shape == b.shape and np.array_equal(a.view(np.uint8), b.view(np.uint8))


def oracle_out(w, act, scale, codes, ws, bias):
    """fp32 reference of the backend with weight width ``w`` (FMA epilogue)."""
    if w == 8:
        return O.tokenwise_linear(act, scale, codes, ws, bias, fma=True)
    return O.rowwise_native_linear(act, scale, codes, ws, bias, fma=True)


def order_of(ops, w):
    return ops.ORDER_TRITON if w == 8 else ops.ORDER_NATIVE


@pytest.mark.parametrize("w", [2, 4, 8])
@pytest.mark.parametrize("si", [0, 1, 2])
def test_wxa4_golden(ops, g, w, si):
    key = f"w{w}_s{si}"
    x = bf16_tensor(g[f"{key}_x"]).to(DEV)
    packed, scale = ops.quantize_rows_a4(x)
    assert bits_equal(packed.cpu().numpy(), g[f"{key}_packed"]) and bits_equal(scale.cpu().numpy(), g[f"{key}_scale"])
    codes = g[f"{key}_codes"]
    rows = ops.pack_rows(torch.from_numpy(codes).to(DEV), w)
    ws = torch.from_numpy(g[f"{key}_ws"]).to(DEV)
    has_bias = f"{key}_bias" in g
    bias_np = g[f"{key}_bias"] if has_bias else None
    bias = torch.from_numpy(bias_np).to(DEV) if has_bias else None
    k = x.shape[1]
    ref = oracle_out(w, g[f"{key}_act"], g[f"{key}_scale"], codes, g[f"{key}_ws"], bias_np)
    for variant in (0, 1, 2, 3, 12, 13):  # AUTO, BN32/64/128, persistent BN64P/BN128P
        y = ops.rowwise_linear(packed, 4, scale, rows, w, ws, bias, k, order=order_of(ops, w),
                               out_dtype=torch.float32, variant=variant)
        assert bits_equal(y.cpu().numpy(), ref), f"fp32 variant {variant}"
        yb = ops.rowwise_linear(packed, 4, scale, rows, w, ws, bias, k, order=order_of(ops, w),
                                out_dtype=torch.bfloat16, variant=variant)
        ours = yb.view(torch.int16).cpu().numpy().view(np.uint16)
        assert bits_equal(ours, O.to_bf16_bits(ref)), f"bf16 variant {variant}"
        if w == 8:
            gold = O.to_bf16_bits(g[f"{key}_out"]).astype(np.int32)
            assert np.abs(ours.astype(np.int32) - gold).max() <= 1


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("k", [64, 2048, 8192, 16384])
def test_rows_a4_quantizer_formula(ops, dtype, k):
    """scale = max(absmax, 1e-8) * fp32(1/7); codes = clamp(round(x / scale), -8, 7),
    even k in the low nibble, for every register-cache size and the re-reading path."""
    torch.manual_seed(k + 1)
    x = (torch.randn(9, k, device=DEV) * 3).to(dtype)
    x[1] = 0
    x[2, 7] = 1e4 if dtype != torch.float16 else 6e4
    packed, scale = ops.quantize_rows_a4(x)
    xf = x.float()
    ref_scale = xf.abs().amax(1).clamp_min(1e-8) * torch.tensor(1.0 / 7.0, dtype=torch.float32)
    assert torch.equal(scale, ref_scale)
    q = torch.round(xf / ref_scale[:, None]).clamp(-8, 7).to(torch.int16) & 15
    ref = (q[:, 0::2] | (q[:, 1::2] << 4)).to(torch.uint8)
    assert torch.equal(packed, ref)


@pytest.mark.parametrize("w", [2, 4, 8])
def test_modules_match_reference_buffers_and_outputs(g, w):
    from actune_b200.kernels import wxa4_native as M
    cls = {2: M.W2A4NativeLinear, 4: M.W4A4NativeLinear, 8: M.W8A4NativeLinear}[w]
    for si in range(3):
        key = f"w{w}_s{si}"
        wt = bf16_tensor(g[f"{key}_weight"])
        n, k = wt.shape
        has_bias = f"{key}_bias" in g
        lin = torch.nn.Linear(k, n, bias=has_bias, device=DEV, dtype=torch.bfloat16)
        with torch.no_grad():
            lin.weight.copy_(wt.to(DEV))
            if has_bias:
                lin.bias.copy_(torch.from_numpy(g[f"{key}_bias"]).to(DEV).bfloat16())
        layer = cls(lin)
        buf = layer.weight_int8 if w == 8 else layer.packed_weight
        assert bits_equal(buf.cpu().numpy(), g[f"{key}_wbuf"])
        assert bits_equal(layer.weight_scale.cpu().numpy(), g[f"{key}_ws"])
        if has_bias:
            assert bits_equal(layer.bias.cpu().numpy(), g[f"{key}_bias"])
        else:
            assert layer.bias.numel() == 0 and layer.bias.dtype == torch.float32
        x = bf16_tensor(g[f"{key}_x"]).to(DEV)
        y = layer(x)
        assert y.dtype == torch.bfloat16 and y.shape == (x.shape[0], n)
        ref = oracle_out(w, g[f"{key}_act"], g[f"{key}_scale"], g[f"{key}_codes"], g[f"{key}_ws"],
                         g[f"{key}_bias"] if has_bias else None)
        assert bits_equal(y.view(torch.int16).cpu().numpy().view(np.uint16), O.to_bf16_bits(ref))
        # fp32 inputs give fp32 outputs (the reference's output template is the input).
        y32 = layer(x.float())
        assert y32.dtype == torch.float32
        other = cls(torch.nn.Linear(k, n, bias=has_bias, device=DEV, dtype=torch.bfloat16))
        other.load_state_dict(layer.state_dict())
        assert torch.equal(other(x), y)
        assert "_rows" not in layer.state_dict()


def test_shared_a4_cache_between_siblings():
    from actune_b200.kernels import wxa4_native as M
    from actune_b200.kernels.w4a8_triton import shared_a8_cache_scope
    torch.manual_seed(0)
    q = M.W4A4NativeLinear(torch.nn.Linear(256, 64, device=DEV, dtype=torch.bfloat16))
    k = M.W2A4NativeLinear(torch.nn.Linear(256, 32, device=DEV, dtype=torch.bfloat16))
    v = M.W8A4NativeLinear(torch.nn.Linear(256, 48, device=DEV, dtype=torch.bfloat16))
    x = torch.randn(5, 256, device=DEV, dtype=torch.bfloat16)
    with shared_a8_cache_scope() as stats:
        a, b, c = q(x), k(x), v(x)
        entry = stats.a4_entry
        assert entry is not None and entry.source is x
        packed = entry.packed
        q(x)
        assert stats.a4_entry.packed is packed
    assert torch.equal(a, q(x)) and torch.equal(b, k(x)) and torch.equal(c, v(x))
    with shared_a8_cache_scope(enabled=False) as stats:
        q(x)
        assert stats.a4_entry is None


def test_wxa4_full_size_rows(ops):
    """M=600, K=4096, N=12288 through the tensor-core GEMM: sampled rows bit-exact in
    fp32 against the oracle for both epilogue orders."""
    torch.manual_seed(5)
    m, k, n = 600, 4096, 12288
    x = torch.randn(m, k, device=DEV, dtype=torch.bfloat16)
    packed, scale = ops.quantize_rows_a4(x)
    act = O.unpack_a4(packed.cpu().numpy())
    rows = [0, 127, 128, 511, 599]
    for w in (4, 8):
        lo, hi = {4: (-8, 8), 8: (-128, 128)}[w]
        codes = torch.randint(lo, hi, (n, k), device=DEV, dtype=torch.int8)
        ws = torch.rand(n, device=DEV) * 0.01
        y = ops.rowwise_linear(packed, 4, scale, ops.pack_rows(codes, w), w, ws, None, k, order=order_of(ops, w),
                               out_dtype=torch.float32)
        ref = oracle_out(w, act[rows], scale.cpu().numpy()[rows], codes.cpu().numpy(), ws.cpu().numpy(), None)
        assert bits_equal(y.cpu().numpy()[rows], ref), w


@pytest.mark.parametrize("w", [2, 4, 8])
@pytest.mark.parametrize("m", [1, 4, 9, 16])
def test_wxa4_decode_sizes(ops, w, m):
    """M <= 16 runs the weight-streaming kernel: fp32 outputs bit-exact against the
    oracle in both epilogue orders, with and without bias, ragged N and a partial
    last K stage (K = 1536) and packed rows that are not whole
    128-byte blocks (K = 1088)."""
    torch.manual_seed(w * 100 + m + 7)
    for k, n, with_bias in ((4096, 4096, True), (1536, 200, False), (1088, 136, True)):
        x = torch.randn(m, k, device=DEV, dtype=torch.bfloat16)
        lo, hi = {4: (-8, 8), 8: (-128, 128), 2: (-2, 2)}[w]
        codes = torch.randint(lo, hi, (n, k), device=DEV, dtype=torch.int8)
        ws = torch.rand(n, device=DEV) * 0.01
        bias = (torch.randn(n, device=DEV) * 0.1) if with_bias else None
        packed, scale = ops.quantize_rows_a4(x)
        act = O.unpack_a4(packed.cpu().numpy())
        for order in (ops.ORDER_TRITON, ops.ORDER_NATIVE):
            y = ops.rowwise_linear(packed, 4, scale, ops.pack_rows(codes, w), w, ws, bias, k, order=order,
                                   out_dtype=torch.float32)
            b = None if bias is None else bias.cpu().numpy()
            fn = O.tokenwise_linear if order == ops.ORDER_TRITON else O.rowwise_native_linear
            ref = fn(act, scale.cpu().numpy(), codes.cpu().numpy(), ws.cpu().numpy(), b, fma=True)
            assert bits_equal(y.cpu().numpy(), ref), (k, n, order)


def test_rowwise_rejects_bad_arguments(ops):
    from actune_b200 import _lib
    a = torch.zeros(4, 128, device=DEV, dtype=torch.uint8)
    s = torch.ones(4, device=DEV)
    w = torch.zeros(8, 128, device=DEV, dtype=torch.uint8)
    ws = torch.ones(8, device=DEV)
    with pytest.raises(_lib.ActuneError):
        ops.rowwise_linear(a, 4, s, w, 4, ws, None, 256, order=2)
    with pytest.raises(RuntimeError):
        ops.rowwise_linear(a, 2, s, w, 4, ws, None, 256)
