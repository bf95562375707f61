"""Tokenwise W{4,8,2}A8 backends on the GPU against the oracle and the reference's goldens.

The goldens (tests/golden/tokenwise.npz, made by tests/golden/gen_tokenwise.py)
come from the reference's own kernels run under the Triton interpreter with fp32
outputs; the oracle (oracle/group64.c) reproduces them bit for bit
(tests/test_oracle.py).  The GPU path computes the epilogue with a fused multiply-
add, as the reference's GPU kernels do, so fp32 outputs are compared with the
oracle's FMA mode bit for bit, and bf16 outputs with the goldens to one bf16 ulp.
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
def tw():
    return np.load(GOLDEN / "tokenwise.npz")


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


@pytest.mark.parametrize("w", [4, 8, 2])
@pytest.mark.parametrize("si", [0, 1, 2])
def test_tokenwise_golden(ops, tw, w, si):
    key = f"w{w}_s{si}"
    x = bf16_tensor(tw[f"{key}_x"]).to(DEV)
    act, scale = ops.quantize_rows_a8(x)
    assert bits_equal(act.cpu().numpy(), tw[f"{key}_act"]) and bits_equal(scale.cpu().numpy(), tw[f"{key}_scale"])
    codes = torch.from_numpy(tw[f"{key}_codes"]).to(DEV)
    rows = ops.pack_rows(codes, w)
    ws = torch.from_numpy(tw[f"{key}_ws"]).to(DEV)
    has_bias = f"{key}_bias" in tw
    bias = bf16_tensor(tw[f"{key}_bias"]).to(DEV) if has_bias else None
    k = x.shape[1]
    ref = O.tokenwise_linear(tw[f"{key}_act"], tw[f"{key}_scale"], tw[f"{key}_codes"], tw[f"{key}_ws"],
                             O.bf16_bits_to_f32(tw[f"{key}_bias"]) if has_bias else None, fma=True)
    for variant in (0, 1, 2, 3, 12, 13):  # AUTO, BN32/64/128, persistent BN64P/BN128P
        y = ops.tokenwise_linear(act, scale, rows, ws, bias, k, w, out_dtype=torch.float32, variant=variant)
        assert bits_equal(y.cpu().numpy(), ref), f"fp32 variant {variant}"
        yb = ops.tokenwise_linear(act, scale, rows, ws, bias, k, w, out_dtype=torch.bfloat16, variant=variant)
        ours = yb.view(torch.int16).cpu().numpy().view(np.uint16).astype(np.int32)
        gold = O.to_bf16_bits(tw[f"{key}_out"]).astype(np.int32)
        assert np.abs(ours - gold).max() <= 1, f"bf16 variant {variant}"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("k", [64, 2048, 8192, 16384])
def test_rows_quantizer_formula(ops, dtype, k):
    """scale = max(absmax, 1e-8) * fp32(1/127); codes = clamp(round(x / scale)) for every
    register-cache size and the re-reading path (K > 8192)."""
    torch.manual_seed(k)
    x = (torch.randn(9, k, device=DEV) * 3).to(dtype)
    x[1] = 0
    x[2, 7] = 1e4 if dtype != torch.float16 else 6e4
    act, scale = ops.quantize_rows_a8(x)
    xf = x.float()
    ref_scale = xf.abs().amax(1).clamp_min(1e-8) * torch.tensor(1.0 / 127.0, dtype=torch.float32)
    assert torch.equal(scale, ref_scale)
    ref_act = torch.round(xf / ref_scale[:, None]).clamp(-128, 127).to(torch.int8)
    assert torch.equal(act, ref_act)


@pytest.mark.parametrize("w", [4, 8, 2])
def test_modules_match_reference_buffers_and_outputs(tw, w):
    from actune_b200.kernels import w2a8_triton, w4a8_triton, w8a8_triton
    cls = {4: w4a8_triton.W4A8TritonLinear, 8: w8a8_triton.W8A8TritonLinear, 2: w2a8_triton.W2A8TritonLinear}[w]
    for si in range(3):
        key = f"w{w}_s{si}"
        wt = bf16_tensor(tw[f"{key}_weight"])
        n, k = wt.shape
        has_bias = f"{key}_bias" in tw
        lin = torch.nn.Linear(k, n, bias=has_bias, device=DEV, dtype=torch.bfloat16)
        with torch.no_grad():
            lin.weight.copy_(wt.to(DEV))
            if has_bias:
                lin.bias.copy_(bf16_tensor(tw[f"{key}_bias"]).to(DEV))
        layer = cls(lin)
        buf = layer.weight_int8 if w == 8 else layer.packed_weight
        assert bits_equal(buf.cpu().numpy(), tw[f"{key}_wbuf"])
        assert bits_equal(layer.weight_scale.cpu().numpy(), tw[f"{key}_ws"])
        x = bf16_tensor(tw[f"{key}_x"]).to(DEV)
        y = layer(x)
        assert y.dtype == torch.bfloat16 and y.shape == (x.shape[0], n)
        ours = y.view(torch.int16).cpu().numpy().view(np.uint16).astype(np.int32)
        gold = O.to_bf16_bits(tw[f"{key}_out"]).astype(np.int32)
        assert np.abs(ours - gold).max() <= 1
        # A state dict loaded into a module built from other weights gives the same layer.
        other = cls(torch.nn.Linear(k, n, bias=has_bias, device=DEV, dtype=torch.bfloat16))
        other.load_state_dict(layer.state_dict())
        assert torch.equal(other(x), y)
        assert "_rows" not in layer.state_dict()


def test_shared_a8_cache_and_replace():
    from actune_b200.kernels import w4a8_triton as M
    torch.manual_seed(0)
    model = torch.nn.Sequential(torch.nn.Linear(256, 128), torch.nn.Linear(128, 64)).to(DEV).bfloat16()
    assert M.replace_with_w4a8_triton_(model, lambda m, name: isinstance(m, torch.nn.Linear)) == 2
    q = M.W4A8TritonLinear(torch.nn.Linear(256, 64, device=DEV, dtype=torch.bfloat16))
    k = M.W4A8TritonLinear(torch.nn.Linear(256, 32, device=DEV, dtype=torch.bfloat16))
    x = torch.randn(5, 256, device=DEV, dtype=torch.bfloat16)
    with M.shared_a8_cache_scope() as stats:
        a, b = q(x), k(x)
    assert (stats.hits, stats.misses) == (1, 1)
    assert torch.equal(a, q(x)) and torch.equal(b, k(x))
    assert model(x).shape == (5, 64)


def test_tokenwise_full_size_rows(ops):
    """The bench-sized W4A8 shape (M=600, K=4096, N=12288): sampled rows bit-exact in
    fp32 against the oracle (rows are independent)."""
    torch.manual_seed(3)
    m, k, n = 600, 4096, 12288
    x = torch.randn(m, k, device=DEV, dtype=torch.bfloat16)
    codes = torch.randint(-8, 8, (n, k), device=DEV, dtype=torch.int8)
    ws = torch.rand(n, device=DEV) * 0.01
    act, scale = ops.quantize_rows_a8(x)
    y = ops.tokenwise_linear(act, scale, ops.pack_rows(codes, 4), ws, None, k, 4, out_dtype=torch.float32)
    rows = [0, 127, 128, 511, 599]
    ref = O.tokenwise_linear(act.cpu().numpy()[rows], scale.cpu().numpy()[rows], codes.cpu().numpy(),
                             ws.cpu().numpy(), None, fma=True)
    assert bits_equal(y.cpu().numpy()[rows], ref)


def test_tokenwise_rejects_bad_arguments(ops):
    from actune_b200 import _lib
    a = torch.zeros(4, 96, device=DEV, dtype=torch.int8)
    s = torch.ones(4, device=DEV)
    w = torch.zeros(8, 48, device=DEV, dtype=torch.uint8)
    ws = torch.ones(8, device=DEV)
    with pytest.raises(_lib.ActuneError):
        ops.tokenwise_linear(a, s, w, ws, None, 96, 4)  # K % 64 != 0


@pytest.mark.parametrize("w", [4, 8, 2])
@pytest.mark.parametrize("m", [1, 4, 9, 16])
def test_tokenwise_decode_sizes(ops, w, m):
    """M <= 16 runs the weight-streaming kernel in its tokenwise mode: fp32 outputs
    bit-exact against the oracle, with and without bias, ragged N and a partial
    last K stage (K = 1536) and packed rows that are not whole
    128-byte blocks (K = 1088)."""
    torch.manual_seed(w * 100 + m)
    for k, n, with_bias in ((4096, 4096, True), (1536, 200, False), (1088, 136, True)):
        x = torch.randn(m, k, device=DEV, dtype=torch.bfloat16)
        lo, hi = {4: (-8, 8), 8: (-128, 128), 2: (-2, 2)}[w]
        codes = torch.randint(lo, hi, (n, k), device=DEV, dtype=torch.int8)
        ws = torch.rand(n, device=DEV) * 0.01
        bias = (torch.randn(n, device=DEV) * 0.1).bfloat16() if with_bias else None
        act, scale = ops.quantize_rows_a8(x)
        y = ops.tokenwise_linear(act, scale, ops.pack_rows(codes, w), ws, bias, k, w, out_dtype=torch.float32)
        ref = O.tokenwise_linear(act.cpu().numpy(), scale.cpu().numpy(), codes.cpu().numpy(), ws.cpu().numpy(),
                                 None if bias is None else bias.float().cpu().numpy(), fma=True)
        assert bits_equal(y.cpu().numpy(), ref), (k, n)


@pytest.mark.parametrize("w", [4, 8, 2])
@pytest.mark.parametrize("n", [4096, 3990])
def test_tokenwise_auto_split_waves(ops, w, n):
    """At M=600 the 128-column tiles leave a partial last wave: AUTO runs the rest of
    the columns as a dependent launch of narrower tiles, identical to the one-launch
    BN128 kernel."""
    torch.manual_seed(n + w)
    m, k = 600, 256
    x = torch.randn(m, k, device=DEV, dtype=torch.bfloat16)
    lo, hi = {4: (-8, 8), 8: (-128, 128), 2: (-2, 2)}[w]
    rows = ops.pack_rows(torch.randint(lo, hi, (n, k), device=DEV, dtype=torch.int8), w)
    ws = torch.rand(n, device=DEV) * 0.01
    bias = (torch.randn(n, device=DEV) * 0.1).bfloat16()
    act, scale = ops.quantize_rows_a8(x)
    auto = ops.tokenwise_linear(act, scale, rows, ws, bias, k, w, variant=0)
    whole = ops.tokenwise_linear(act, scale, rows, ws, bias, k, w, variant=3)
    assert torch.equal(auto, whole)
