"""Torch-tensor face of the C ABI: allocation, shape checks, device/stream plumbing.

Every function here ends in exactly one C-ABI call on the tensor's device and
current stream; nothing computes on the host.  Errors follow the reference's
conventions: wrong devices/shapes/dtypes raise RuntimeError (the reference's
TORCH_CHECKs, actune/kernels/grouped_native.cu:92-105), and a non-zero status
from the library raises ``actune_b200._lib.ActuneError`` (a RuntimeError).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

_DTYPES = {torch.float32: _lib.DTYPE_F32, torch.float16: _lib.DTYPE_F16, torch.bfloat16: _lib.DTYPE_BF16}


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPES[dtype]
    except KeyError:
        raise RuntimeError(f"unsupported dtype {dtype} (float32, float16 or bfloat16 required)") from None


def _ptr(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _stream(device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _require(cond, msg):
    if not cond:
        raise RuntimeError(msg)


def _cuda_contig(*tensors):
    dev = None
    for t in tensors:
        if t is None:
            continue
        _require(t.is_cuda, "CUDA required")
        _require(t.is_contiguous(), "contiguous operands required")
        dev = t.device if dev is None else dev
        _require(t.device == dev, "device mismatch")
    return dev


def quantize_group64(x: torch.Tensor, bits: int, packed: torch.Tensor | None = None,
                     scales: torch.Tensor | None = None, codes8: bool = False):
    """Group-64 activation quantizer: x [M, K] -> (packed u8 [M, K*bits/8], scales f32 [M, K/64]).
    ``codes8``: the same codes one byte each, u8 [M, K] (the A=8 operand layout)."""
    _require(x.dim() == 2, "x must be 2-D [M, K]")
    m, k = x.shape
    _require(bits in (2, 4, 8), "Unsupported integer width")
    _require(k % 64 == 0, "K must be a multiple of 64")
    width = 8 if codes8 else bits
    if packed is None:
        packed = torch.empty((m, k * width // 8), device=x.device, dtype=torch.uint8)
    if scales is None:
        scales = torch.empty((m, k // 64), device=x.device, dtype=torch.float32)
    dev = _cuda_contig(x, packed, scales)
    entry = _lib.lib().actune_quantize_group64_codes if codes8 else _lib.lib().actune_quantize_group64
    with torch.cuda.device(dev):
        _lib.check(entry(_ptr(x), dtype_code(x.dtype), m, k, bits, _ptr(packed), _ptr(scales), _stream(dev)),
                   "quantize_group64")
    return packed, scales


def packed_linear(a, a_scale, w, w_scale, bias, K: int, W: int, A: int, out_dtype=torch.bfloat16,
                  variant: int = _lib.VARIANT_AUTO, out: torch.Tensor | None = None):
    """out[M, N] = ws * sum_g float(dot_g) * as[:, g] (+ bias), exact reference fp32 order."""
    _require(a.dim() == 2 and w.dim() == 2, "rank mismatch")
    m, n = a.shape[0], w.shape[0]
    _require(a.dtype == torch.uint8 and w.dtype == torch.uint8, "packed uint8 required")
    _require(a_scale.dtype == torch.float32 and w_scale.dtype == torch.float32, "float scales required")
    _require(K % 64 == 0 and K > 0, "invalid dimensions")
    _require(a.shape[1] == K * A // 8 and w.shape[1] == K * W // 8, "packed shape mismatch")
    _require(tuple(a_scale.shape) == (m, K // 64) and w_scale.numel() == n, "scale shape mismatch")
    if bias is not None and bias.numel() == 0:
        bias = None
    _require(bias is None or bias.numel() == n, "bias shape mismatch")
    if out is None:
        out = torch.empty((m, n), device=a.device, dtype=out_dtype)
    _require(tuple(out.shape) == (m, n), "output shape mismatch")
    dev = _cuda_contig(a, a_scale, w, w_scale, bias, out)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().actune_packed_linear(
            _ptr(a), _ptr(a_scale), _ptr(w), _ptr(w_scale), _ptr(bias),
            _lib.DTYPE_NONE if bias is None else dtype_code(bias.dtype), _ptr(out), dtype_code(out.dtype),
            m, n, K, W, A, int(variant), _stream(dev)), "packed_linear")
    return out


def quantize_rows_a8(x, codes=None, scales=None):
    """Per-row dynamic INT8 activations of x [M, K]: (codes int8 [M, K], scales f32 [M]),
    scale = max(row absmax, 1e-8) * fp32(1/127), reference w4a8_triton.py:161-201."""
    _require(x.dim() == 2, "x must be 2-D [M, K]")
    m, k = x.shape
    _require(k % 8 == 0, "K must be a multiple of 8")
    if codes is None:
        codes = torch.empty((m, k), device=x.device, dtype=torch.int8)
    if scales is None:
        scales = torch.empty(m, device=x.device, dtype=torch.float32)
    dev = _cuda_contig(x, codes, scales)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().actune_quantize_rows_a8(_ptr(x), dtype_code(x.dtype), m, k, _ptr(codes), _ptr(scales),
                                                      _stream(dev)), "quantize_rows_a8")
    return codes, scales


def tokenwise_linear(a, a_scale, w_rows, w_scale, bias, K: int, W: int, out_dtype=torch.bfloat16,
                     variant: int = _lib.VARIANT_AUTO, out: torch.Tensor | None = None):
    """out[M, N] = float(a @ codes.T) * a_scale[:, None] * w_scale (+ bias) for int8
    activations [M, K] and weight codes packed as rows [N, K*W/8]."""
    _require(a.dim() == 2 and w_rows.dim() == 2, "rank mismatch")
    m, n = a.shape[0], w_rows.shape[0]
    _require(a.dtype == torch.int8 and w_rows.dtype == torch.uint8, "int8 activations and uint8 weight rows required")
    _require(a.shape[1] == K and w_rows.shape[1] == K * W // 8, "packed shape mismatch")
    _require(a_scale.numel() == m and w_scale.numel() == n, "scale shape mismatch")
    if bias is not None and bias.numel() == 0:
        bias = None
    if out is None:
        out = torch.empty((m, n), device=a.device, dtype=out_dtype)
    dev = _cuda_contig(a, a_scale, w_rows, w_scale, bias, out)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().actune_tokenwise_linear(
            _ptr(a), _ptr(a_scale), _ptr(w_rows), _ptr(w_scale), _ptr(bias),
            _lib.DTYPE_NONE if bias is None else dtype_code(bias.dtype), _ptr(out), dtype_code(out.dtype),
            m, n, K, W, int(variant), _stream(dev)), "tokenwise_linear")
    return out


def quantize_rows_a4(x, packed=None, scales=None):
    """Per-row dynamic INT4 activations of x [M, K]: (packed u8 [M, K/2] with even k in
    the low nibble, scales f32 [M]), scale = max(row absmax, 1e-8) * fp32(1/7),
    reference wxa4_native.py:27-64."""
    _require(x.dim() == 2, "x must be 2-D [M, K]")
    m, k = x.shape
    _require(k % 8 == 0, "K must be a multiple of 8")
    if packed is None:
        packed = torch.empty((m, k // 2), device=x.device, dtype=torch.uint8)
    if scales is None:
        scales = torch.empty(m, device=x.device, dtype=torch.float32)
    dev = _cuda_contig(x, packed, scales)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().actune_quantize_rows_a4(_ptr(x), dtype_code(x.dtype), m, k, _ptr(packed), _ptr(scales),
                                                      _stream(dev)), "quantize_rows_a4")
    return packed, scales


ORDER_TRITON = 0   # (float(acc) * as) * ws (+ bias): the Triton tokenwise kernels
ORDER_NATIVE = 1   # float(acc) * (as * ws) (+ bias): the native S4 CUDA kernels


def rowwise_linear(a, A: int, a_scale, w_rows, W: int, w_scale, bias, K: int, order: int = ORDER_TRITON,
                   out_dtype=torch.bfloat16, variant: int = _lib.VARIANT_AUTO, out: torch.Tensor | None = None):
    """Row-scaled linear for A-bit activation rows [M, K*A/8] (A = 8 int8 codes, A = 4
    packed nibbles) and W-bit weight rows [N, K*W/8]: exact int32 dots over all of K,
    one scale per token and per output channel, epilogue in ``order``."""
    _require(a.dim() == 2 and w_rows.dim() == 2, "rank mismatch")
    _require(A in (4, 8) and W in (2, 4, 8), "Unsupported integer width")
    m, n = a.shape[0], w_rows.shape[0]
    _require(a.dtype in (torch.uint8, torch.int8) and w_rows.dtype == torch.uint8, "packed uint8 rows required")
    _require(a.shape[1] == K * A // 8 and w_rows.shape[1] == K * W // 8, "packed shape mismatch")
    _require(a_scale.numel() == m and w_scale.numel() == n, "scale shape mismatch")
    _require(a_scale.dtype == torch.float32 and w_scale.dtype == torch.float32, "float scales required")
    if bias is not None and bias.numel() == 0:
        bias = None
    if out is None:
        out = torch.empty((m, n), device=a.device, dtype=out_dtype)
    dev = _cuda_contig(a, a_scale, w_rows, w_scale, bias, out)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().actune_rowwise_linear(
            _ptr(a), A, _ptr(a_scale), _ptr(w_rows), W, _ptr(w_scale), _ptr(bias),
            _lib.DTYPE_NONE if bias is None else dtype_code(bias.dtype), _ptr(out), dtype_code(out.dtype),
            m, n, K, int(order), int(variant), _stream(dev)), "rowwise_linear")
    return out


def packed_linear_dots(a, w, K: int, W: int, A: int, variant: int = _lib.VARIANT_AUTO):
    """Exact per-group int32 dots [M, N, K/64] from the tensor-core kernel (debug export)."""
    m, n = a.shape[0], w.shape[0]
    _require(a.shape[1] == K * A // 8 and w.shape[1] == K * W // 8, "packed shape mismatch")
    dots = torch.empty((m, n, K // 64), device=a.device, dtype=torch.int32)
    dev = _cuda_contig(a, w, dots)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().actune_packed_linear_dots(_ptr(a), _ptr(w), _ptr(dots), m, n, K, W, A, int(variant),
                                                        _stream(dev)), "packed_linear_dots")
    return dots


def weight_codes(weight: torch.Tensor, W: int, A: int, clip: torch.Tensor | None = None):
    """Per-row codebook on the GPU: (codes int8 [N, K], scale f32 [N])."""
    _require(weight.dim() == 2, "weight must be 2-D [N, K]")
    n, k = weight.shape
    codes = torch.empty((n, k), device=weight.device, dtype=torch.int8)
    scale = torch.empty((n,), device=weight.device, dtype=torch.float32)
    if clip is not None:
        clip = clip.to(device=weight.device, dtype=torch.float32).contiguous()
    dev = _cuda_contig(weight, clip, codes, scale)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().actune_weight_codes(_ptr(weight), dtype_code(weight.dtype), n, k, W, A, _ptr(clip),
                                                  _ptr(codes), _ptr(scale), _stream(dev)), "weight_codes")
    return codes, scale


def r4_refine(weight: torch.Tensor, q4: torch.Tensor, scale4: torch.Tensor):
    """Nested W8 residual for given int4 codes/scales: (residual int8, q8 int8)."""
    _require(weight.dim() == 2 and q4.shape == weight.shape, "q4 must match weight [N, K]")
    n, k = weight.shape
    q4 = q4.to(device=weight.device, dtype=torch.int8).contiguous()
    scale4 = scale4.to(device=weight.device, dtype=torch.float32).contiguous()
    residual = torch.empty((n, k), device=weight.device, dtype=torch.int8)
    q8 = torch.empty((n, k), device=weight.device, dtype=torch.int8)
    dev = _cuda_contig(weight, q4, scale4, residual, q8)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().actune_r4_refine(_ptr(weight), dtype_code(weight.dtype), n, k, _ptr(q4), _ptr(scale4),
                                               _ptr(residual), _ptr(q8), _stream(dev)), "r4_refine")
    return residual, q8


def pack_rows(q: torch.Tensor, bits: int):
    """Little-endian sub-byte packing of int8 codes [R, K] -> uint8 [R, K*bits/8]."""
    _require(q.dim() == 2 and q.dtype == torch.int8, "int8 [R, K] codes required")
    r, k = q.shape
    _require(bits in (2, 4, 8) and k % (8 // bits) == 0, "K must be a multiple of 8/bits")
    packed = torch.empty((r, k * bits // 8), device=q.device, dtype=torch.uint8)
    dev = _cuda_contig(q, packed)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().actune_pack_rows(_ptr(q), r, k, bits, _ptr(packed), _stream(dev)), "pack_rows")
    return packed


def workspace_size(M: int, K: int, A: int) -> int:
    return int(_lib.lib().actune_grouped_linear_workspace_size(M, K, A))


def grouped_linear(x, w, w_scale, bias, W: int, A: int, workspace: torch.Tensor | None = None,
                   variant: int = _lib.VARIANT_AUTO, out: torch.Tensor | None = None):
    """One-call quantize + packed GEMM for x [M, K] (caller-provided workspace)."""
    _require(x.dim() == 2, "x must be 2-D [M, K]")
    m, k = x.shape
    n = w.shape[0]
    if bias is not None and bias.numel() == 0:
        bias = None
    need = workspace_size(m, k, A)
    if workspace is None:
        workspace = torch.empty((max(need, 1),), device=x.device, dtype=torch.uint8)
    if out is None:
        out = torch.empty((m, n), device=x.device, dtype=x.dtype)
    dev = _cuda_contig(x, w, w_scale, bias, out, workspace)
    with torch.cuda.device(dev):
        _lib.check(_lib.lib().actune_grouped_linear(
            _ptr(x), dtype_code(x.dtype), m, k, _ptr(w), _ptr(w_scale), _ptr(bias),
            _lib.DTYPE_NONE if bias is None else dtype_code(bias.dtype), n, W, A, _ptr(out), dtype_code(out.dtype),
            _ptr(workspace), workspace.numel() * workspace.element_size(), int(variant), _stream(dev)),
            "grouped_linear")
    return out
