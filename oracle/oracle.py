"""Python face of the CPU oracle.  TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import
this module; the product package ``actune_b200`` never does.  Every function is
a checker, never the thing shipped or measured as the product.

Two parts:

* ctypes bindings of ``group64.c`` (the bit-exact restatement of the reference's
  integer path: activation quantizer, weight codebooks, pack, per-group int32
  dots, fp32 epilogue), numpy in / numpy out;
* ``dequant_linear``: the reference's CPU dequantize-and-matmul formula,
  ``F.linear(activation_reference(x, a), q.float() * scale[:, None], bias)``
  (reference tests/test_kernels.py:42-44 with actune/calibration.py:7-16), in
  torch on the host cores.  It is the timed CPU baseline; it is *not* bit-exact
  with the integer path (fp32 GEMM summation order differs), which is why the
  reference's own test compares it at rtol=atol=0.02.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle_group64.so"
_LIB = None


def build(force: bool = False) -> Path:
    """Compile group64.c with the committed Makefile (no-op when up to date)."""
    if force or not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < (HERE / "group64.c").stat().st_mtime:
        env = dict(os.environ)
        env.setdefault("CC", "gcc")
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True, env=env)
    return LIB_PATH


def lib():
    global _LIB
    if _LIB is None:
        build()
        L = ctypes.CDLL(str(LIB_PATH))
        i64, i32, p = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p
        L.oracle_quantize_group64_bf16.argtypes = [p, i64, i64, i32, p, p]
        L.oracle_quantize_group64_f32.argtypes = [p, i64, i64, i32, p, p]
        L.oracle_unpack_rows.argtypes = [p, i64, i64, i32, p]
        L.oracle_pack_rows.argtypes = [p, i64, i64, i32, p]
        L.oracle_group_dots.argtypes = [p, p, i64, i64, i64, i32, i32, p]
        L.oracle_packed_linear.argtypes = [p, p, p, p, p, i64, i64, i64, i32, i32, i32, p]
        L.oracle_weight_codes.argtypes = [p, i64, i64, i32, i32, p, p, p]
        L.oracle_quantize_rows_a8.argtypes = [p, i64, i64, p, p]
        L.oracle_tokenwise_linear.argtypes = [p, p, p, p, p, i64, i64, i64, i32, p]
        L.oracle_quantize_rows_a4.argtypes = [p, i64, i64, p, p]
        L.oracle_rowwise_native_linear.argtypes = [p, p, p, p, p, i64, i64, i64, i32, p]
        L.oracle_f32_to_bf16_array.argtypes = [p, p, i64]
        L.oracle_f32_to_bf16_array.restype = None
        _LIB = L
    return _LIB


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _check(rc):
    if rc != 0:
        raise ValueError(f"oracle rejected the arguments (status {rc})")


def quantize_group64(x, bits: int):
    """x: [M, K] as uint16 bf16 bits or float32. Returns (packed u8, scales f32)."""
    x = np.ascontiguousarray(x)
    M, K = x.shape
    packed = np.zeros((M, K * bits // 8), np.uint8)
    scales = np.zeros((M, K // 64), np.float32)
    fn = lib().oracle_quantize_group64_bf16 if x.dtype == np.uint16 else lib().oracle_quantize_group64_f32
    if x.dtype not in (np.uint16, np.float32):
        raise TypeError("x must be bf16 bits (uint16) or float32")
    _check(fn(_ptr(x), M, K, bits, _ptr(packed), _ptr(scales)))
    return packed, scales


def unpack_rows(packed, K: int, bits: int):
    packed = np.ascontiguousarray(packed, np.uint8)
    R = packed.shape[0]
    codes = np.zeros((R, K), np.int8)
    _check(lib().oracle_unpack_rows(_ptr(packed), R, K, bits, _ptr(codes)))
    return codes


def pack_rows(q, bits: int):
    q = np.ascontiguousarray(q, np.int8)
    R, K = q.shape
    out = np.zeros((R, K * bits // 8), np.uint8)
    _check(lib().oracle_pack_rows(_ptr(q), R, K, bits, _ptr(out)))
    return out


def group_dots(a, w, K: int, W: int, A: int):
    """Per-64-group int32 dots [M, N, K/64]."""
    a = np.ascontiguousarray(a, np.uint8)
    w = np.ascontiguousarray(w, np.uint8)
    M, N = a.shape[0], w.shape[0]
    dots = np.zeros((M, N, K // 64), np.int32)
    _check(lib().oracle_group_dots(_ptr(a), _ptr(w), M, N, K, W, A, _ptr(dots)))
    return dots


def packed_linear(a, a_scale, w, w_scale, bias, K: int, W: int, A: int, fma: bool = True):
    """fp32 [M, N] output of the reference's integer path (bias may be None)."""
    a = np.ascontiguousarray(a, np.uint8)
    w = np.ascontiguousarray(w, np.uint8)
    a_scale = np.ascontiguousarray(a_scale, np.float32)
    w_scale = np.ascontiguousarray(w_scale, np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    M, N = a.shape[0], w.shape[0]
    out = np.zeros((M, N), np.float32)
    _check(lib().oracle_packed_linear(_ptr(a), _ptr(a_scale), _ptr(w), _ptr(w_scale), _ptr(b),
                                      M, N, K, W, A, 1 if fma else 0, _ptr(out)))
    return out


def weight_codes(weight, W: int, A: int, clip=None):
    """weight: float32 [N, K] (bf16 values widened). Returns (codes int8, scale f32)."""
    weight = np.ascontiguousarray(weight, np.float32)
    N, K = weight.shape
    c = None
    if clip is not None:
        c = np.ascontiguousarray(np.broadcast_to(np.asarray(clip, np.float32).reshape(-1), (N,)), np.float32)
    codes = np.zeros((N, K), np.int8)
    scale = np.zeros((N,), np.float32)
    _check(lib().oracle_weight_codes(_ptr(weight), N, K, W, A, _ptr(c), _ptr(codes), _ptr(scale)))
    return codes, scale


def quantize_rows_a8(x_bf16_bits):
    """Per-row dynamic INT8 codes [M, K] int8 and scales [M] f32 of a bf16 matrix
    (given as uint16 bits), reference w4a8_triton.py:161-201."""
    x = np.ascontiguousarray(x_bf16_bits, np.uint16)
    M, K = x.shape
    codes = np.empty((M, K), np.int8)
    scales = np.empty(M, np.float32)
    _check(lib().oracle_quantize_rows_a8(_ptr(x), M, K, _ptr(codes), _ptr(scales)))
    return codes, scales


def tokenwise_linear(a, a_scale, codes, w_scale, bias, fma: bool = True):
    """Tokenwise W{2,4,8}A8 linear [M, N] f32 from int8 activations [M, K], row
    scales [M], weight codes [N, K] int8 and row scales [N] (reference
    w4a8_triton.py:57-114)."""
    a = np.ascontiguousarray(a, np.int8)
    codes = np.ascontiguousarray(codes, np.int8)
    a_scale = np.ascontiguousarray(a_scale, np.float32)
    w_scale = np.ascontiguousarray(w_scale, np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    M, K = a.shape
    N = codes.shape[0]
    out = np.empty((M, N), np.float32)
    _check(lib().oracle_tokenwise_linear(_ptr(a), _ptr(a_scale), _ptr(codes), _ptr(w_scale), _ptr(b), M, N, K,
                                         1 if fma else 0, _ptr(out)))
    return out


def quantize_rows_a4(x_bf16_bits):
    """Per-row dynamic INT4 activations of a bf16 matrix (uint16 bits): packed [M, K/2]
    u8 (even k in the low nibble) and scales [M] f32 (reference wxa4_native.py:27-64)."""
    x = np.ascontiguousarray(x_bf16_bits, np.uint16)
    M, K = x.shape
    packed = np.empty((M, (K + 1) // 2), np.uint8)
    scales = np.empty(M, np.float32)
    _check(lib().oracle_quantize_rows_a4(_ptr(x), M, K, _ptr(packed), _ptr(scales)))
    return packed, scales


def unpack_a4(packed, K=None):
    """Packed nibble rows [M, K/2] -> signed int8 codes [M, K] (even k low nibble)."""
    p = np.ascontiguousarray(packed, np.uint8).astype(np.int16)
    lo, hi = ((p & 15) ^ 8) - 8, (((p >> 4) & 15) ^ 8) - 8
    out = np.stack([lo, hi], -1).reshape(p.shape[0], -1).astype(np.int8)
    return out if K is None else out[:, :K]


def rowwise_native_linear(a, a_scale, codes, w_scale, bias, fma: bool = True):
    """Native W{2,4}A4 linear [M, N] f32: float(acc) * (as[m] * ws[n]) (+ bias), from
    int8 activation codes [M, K] and weight codes [N, K]
    (reference native_s4_extension_kernel.cu:226-234)."""
    a = np.ascontiguousarray(a, np.int8)
    codes = np.ascontiguousarray(codes, np.int8)
    a_scale = np.ascontiguousarray(a_scale, np.float32)
    w_scale = np.ascontiguousarray(w_scale, np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    M, K = a.shape
    N = codes.shape[0]
    out = np.empty((M, N), np.float32)
    _check(lib().oracle_rowwise_native_linear(_ptr(a), _ptr(a_scale), _ptr(codes), _ptr(w_scale), _ptr(b), M, N, K,
                                              1 if fma else 0, _ptr(out)))
    return out


def to_bf16_bits(x):
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros(x.shape, np.uint16)
    lib().oracle_f32_to_bf16_array(_ptr(x), _ptr(out), x.size)
    return out


def bf16_bits_to_f32(bits):
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------------------
# The reference's CPU dequantize-and-matmul formula (timed CPU baseline).
# ---------------------------------------------------------------------------
def activation_reference(value, bits: int, group_size: int = 64):
    """actune/calibration.py:7-16 restated in torch: fake-quantized activations."""
    import torch
    if bits not in (2, 4, 8) or value.shape[-1] % group_size:
        raise ValueError("Unsupported activation width or unaligned input")
    shape = value.shape
    v = value.float().reshape(*shape[:-1], -1, group_size)
    positive = (1 << (bits - 1)) - 1
    scale = v.abs().amax(-1, keepdim=True).clamp_min(1e-8) / positive
    codes = (v / scale).round().clamp(-positive - 1, positive)
    return (codes * scale).reshape(shape)


def dequant_weight(codes, scale):
    """q.float() * scale[:, None] (hoisted out of the timed region by callers)."""
    return codes.float() * scale[:, None]


def dequant_linear(x, weight_f32, bias, bits: int):
    """F.linear(activation_reference(x, a), dequantized weight, bias) on the CPU."""
    import torch.nn.functional as F
    return F.linear(activation_reference(x, bits), weight_f32, None if bias is None else bias.float())
