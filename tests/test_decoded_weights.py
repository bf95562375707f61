"""Decoded weight codes: the int8 copy of a packed sub-byte version that the tile
GEMM reads for calls of more than 32 token rows.

* CPU: ``unpack_rows`` inverts the reference's little-endian packing (checked
  against the oracle's packer and unpacker for every width, ragged K included).
* GPU: a layer with decoded codes (weights kept as int8 codes, activations
  quantized to the same A-bit codes written one byte each, the W=8 / A=8 kernel)
  gives bit-identical outputs to the packed path for every sub-byte W x A pair, on
  both sides of the 32-row switch, with and without bias; the int8-code quantizer
  writes exactly the unpacked packed codes; the bank runtime reports the bytes it
  added and the storage audit of the packed versions is unchanged.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O


@pytest.mark.parametrize("bits", [2, 4, 8])
@pytest.mark.parametrize("k", [64, 128, 4160])
def test_unpack_rows_inverts_packing(bits, k):
    from actune_b200.kernels.grouped import unpack_rows
    rng = np.random.default_rng(bits * 100 + k)
    lo, hi = -(1 << (bits - 1)), (1 << (bits - 1)) - 1
    codes = rng.integers(lo, hi + 1, size=(7, k), dtype=np.int8)
    packed = O.pack_rows(codes, bits)
    got = unpack_rows(torch.from_numpy(packed), bits, k).numpy()
    assert got.dtype == np.int8
    assert np.array_equal(got, codes)
    assert np.array_equal(got, O.unpack_rows(packed, k, bits))


PAIRS = [(4, 8), (2, 8), (4, 4), (2, 4), (4, 2), (2, 2)]


@pytest.mark.gpu
@pytest.mark.parametrize("w,a", PAIRS)
@pytest.mark.parametrize("bias", [False, True])
def test_decoded_codes_bit_identical_to_packed(w, a, bias):
    from actune_b200.kernels.grouped import DECODED_MIN_TOKENS, GroupedLinear
    torch.manual_seed(w * 10 + a)
    linear = torch.nn.Linear(1024, 320, bias=bias, device="cuda", dtype=torch.bfloat16)
    layer = GroupedLinear(linear, w, a, None)
    xs = {m: torch.randn(m, 1024, device="cuda", dtype=torch.bfloat16) for m in (16, 32, 33, 64, 200, 600)}
    packed_out = {m: layer(x) for m, x in xs.items()}
    added = layer.decode_weight()
    assert added == 320 * 1024 and layer.decoded_weight.dtype == torch.uint8
    assert layer.decode_weight() == 0  # idempotent
    for m, x in xs.items():
        weight, width, a_kernel = layer.operands(m)
        decoded = m >= DECODED_MIN_TOKENS
        assert (width, a_kernel) == ((8, 8) if decoded else (w, a))
        assert layer.activation_format(m) == (a, decoded and a < 8)
        assert torch.equal(layer(x), packed_out[m]), (w, a, m)


@pytest.mark.gpu
@pytest.mark.parametrize("bits", [2, 4, 8])
def test_int8_code_quantizer_is_the_unpacked_packed_one(bits):
    from actune_b200 import ops
    from actune_b200.kernels.grouped import unpack_rows
    torch.manual_seed(bits)
    x = torch.randn(37, 1536, device="cuda", dtype=torch.bfloat16) * 3
    packed, scales = ops.quantize_group64(x, bits)
    codes, scales8 = ops.quantize_group64(x, bits, codes8=True)
    assert codes.shape == (37, 1536) and torch.equal(scales8, scales)
    assert torch.equal(codes.view(torch.int8), unpack_rows(packed, bits, 1536))


@pytest.mark.gpu
def test_runtime_decodes_every_sub_byte_version():
    from actune_b200.harness import make_oft_policy
    from actune_b200.layers import tensor_storage_bytes
    model, runtime = make_oft_policy(layers=2, tokens=64, seed=2, decoded=False)
    storage = {n: tensor_storage_bytes(m) for n, m in runtime.modules.items()}
    x = torch.randn(64, 4096, device="cuda", dtype=torch.bfloat16)
    qkv = runtime.modules["layers.0.qkv_proj"]
    before = qkv(x)
    added = runtime.decode_weights()
    expected = sum(b.out_features * b.in_features for m in runtime.modules.values() for b in m.backends.values()
                   if b.w < 8)
    assert added == expected > 0
    assert runtime.decode_weights() == 0
    assert torch.equal(qkv(x), before)
    assert {n: tensor_storage_bytes(m) for n, m in runtime.modules.items()} == storage
