"""Tokenwise W8A8 backend: drop-in for the reference's actune/kernels/w8a8_triton.py.

``W8A8TritonLinear(linear, fused_quantization=True)`` with buffers ``weight_int8``
int8 [K, N] (K-major, w8a8_triton.py:101-106), ``weight_scale`` f32 [N] and
``bias``; ``replace_with_w8a8_triton_``.  Per-row RTN codes: scale =
max(row absmax, 1e-8) / 127 (IEEE division), codes clamp(round(w / scale),
-128, 127).  The GEMM and activation quantizer are the library's tokenwise entry
points (see w4a8_triton).
"""
from __future__ import annotations

import torch

from ._tokenwise import TokenwiseLinear, replace_with
from .quantizers import weight_codes


class W8A8TritonLinear(TokenwiseLinear):
    """Inference-only Linear with K-major signed-INT8 weights."""

    bits = 8

    def __init__(self, linear: torch.nn.Linear, fused_quantization: bool = True) -> None:
        super().__init__()
        if linear.in_features % 128:
            raise ValueError("in_features must be divisible by 128")
        with torch.no_grad():
            codes, scale = weight_codes(linear.weight, 8, 8)
        self.register_buffer("weight_int8", codes.t().contiguous())
        self.register_buffer("weight_scale", scale.contiguous())
        self._init_common(linear, fused_quantization, codes)

    def _codes_from_buffer(self):
        return self.weight_int8.t().contiguous()


def replace_with_w8a8_triton_(module: torch.nn.Module, filter_fn) -> int:
    """Recursively replace eligible Linear children with W8A8 backends."""
    return replace_with(module, filter_fn, W8A8TritonLinear)
