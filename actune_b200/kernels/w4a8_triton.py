"""Tokenwise W4A8 backend: drop-in for the reference's actune/kernels/w4a8_triton.py.

Same public surface: ``W4A8TritonLinear(linear, fused_quantization=True, *,
weight_clip_ratios=None)`` with buffers ``packed_weight`` u8 [K/2, N] (K-major;
the byte at (j, n) holds the codes of k = j in its low nibble and k = j + K/2 in
its high nibble, w4a8_triton.py:380-383), ``weight_scale`` f32 [N] and ``bias``;
``shared_a8_cache_scope`` / ``clear_shared_a8_cache`` / ``SharedA8CacheStats``;
``replace_with_w4a8_triton_``.  The module name is kept so imports carry over; no
Triton runs here: the activation quantizer and the GEMM are the library's
``actune_quantize_rows_a8`` and ``actune_tokenwise_linear`` (tcgen05, exact INT32
accumulation, the reference's epilogue order).

Weight codes: per-row RTN, scale = max(row absmax, 1e-8) / 7 (IEEE division),
codes clamp(round(w / scale), -8, 7), or the clip-ratio variant of
``quantizers.symmetric_int4_quantize`` (w4a8_triton.py:362-377).
"""
from __future__ import annotations

import torch

from ._tokenwise import (  # noqa: F401  (public names of the reference module)
    SharedA8CacheStats,
    TokenwiseLinear,
    clear_shared_a8_cache,
    quantize_rows_shared as _quantize_rows_shared,
    replace_with,
    shared_a8_cache_scope,
)
from .quantizers import symmetric_int4_quantize


class W4A8TritonLinear(TokenwiseLinear):
    """Inference-only Linear with K-major packed symmetric INT4 weights."""

    bits = 4
    gemv_max_rows = 0

    def __init__(self, linear: torch.nn.Linear, fused_quantization: bool = True, *, weight_clip_ratios=None):
        super().__init__()
        if linear.in_features % 32:
            raise ValueError("in_features must be divisible by 32")
        if linear.in_features % 64:
            raise ValueError("in_features must be divisible by 64 on this backend")
        with torch.no_grad():
            codes, scale = symmetric_int4_quantize(linear.weight, clip_ratios=weight_clip_ratios)
            self.weight_quantizer = ("rtn_per_output_row_v1" if weight_clip_ratios is None
                                     else "awq_style_nested_clip_v1")
            half = linear.in_features // 2
            low = codes[:, :half].to(torch.int16) & 15
            high = (codes[:, half:].to(torch.int16) & 15) << 4
            packed = (low | high).to(torch.uint8).t().contiguous()
        self.register_buffer("packed_weight", packed)
        self.register_buffer("weight_scale", scale.contiguous())
        self._init_common(linear, fused_quantization, codes)

    def _codes_from_buffer(self):
        p = self.packed_weight.t().to(torch.int16)
        low, high = ((p & 15) ^ 8) - 8, (((p >> 4) & 15) ^ 8) - 8
        return torch.cat([low, high], 1).to(torch.int8)


def replace_with_w4a8_triton_(module: torch.nn.Module, filter_fn) -> int:
    """Recursively replace eligible Linear children with W4A8 backends."""
    return replace_with(module, filter_fn, W4A8TritonLinear)
