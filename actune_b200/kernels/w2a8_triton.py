"""Tokenwise W2A8 backend: drop-in for the reference's actune/kernels/w2a8_triton.py.

``W2A8TritonLinear(linear, fused_quantization=True, *, weight_clip_ratios=None)``
with buffers ``packed_weight`` u8 [K/4, N] (K-major; the byte at (j, n) holds the
codes of k = j + i*K/4 in bits 2i..2i+1, w2a8_triton.py:151-159),
``weight_scale`` f32 [N] (the possibly clipped row absmax) and ``bias``;
``replace_with_w2a8_triton_``.  Codes from ``quantizers.symmetric_int2_quantize``
(codebook {-2, -1, 0, 1}).  The GEMM and activation quantizer are the library's
tokenwise entry points (see w4a8_triton).
"""
from __future__ import annotations

import torch

from ._tokenwise import TokenwiseLinear, replace_with
from .quantizers import symmetric_int2_quantize


class W2A8TritonLinear(TokenwiseLinear):
    """Inference-only Linear with K-major packed signed-INT2 weights."""

    bits = 2

    def __init__(self, linear: torch.nn.Linear, fused_quantization: bool = True, *, weight_clip_ratios=None):
        super().__init__()
        if linear.in_features % 128:
            raise ValueError("in_features must be divisible by 128")
        with torch.no_grad():
            codes, scale = symmetric_int2_quantize(linear.weight, clip_ratios=weight_clip_ratios)
            quarter = linear.in_features // 4
            fields = [codes[:, i * quarter:(i + 1) * quarter].to(torch.int16) & 3 for i in range(4)]
            packed = (fields[0] | (fields[1] << 2) | (fields[2] << 4) | (fields[3] << 6)).to(torch.uint8)
            packed = packed.t().contiguous()
        self.register_buffer("packed_weight", packed)
        self.register_buffer("weight_scale", scale.contiguous())
        self.weight_quantizer = ("rtn_per_output_row_w2_v1" if weight_clip_ratios is None
                                 else "awq_style_joint_precision_lattice_clip_v1")
        self._init_common(linear, fused_quantization, codes)

    def _codes_from_buffer(self):
        p = self.packed_weight.t().to(torch.int16)
        return torch.cat([(((p >> (2 * i)) & 3) ^ 2) - 2 for i in range(4)], 1).to(torch.int8)


def replace_with_w2a8_triton_(module: torch.nn.Module, filter_fn) -> int:
    """Recursively replace eligible Linear children with W2A8 backends."""
    return replace_with(module, filter_fn, W2A8TritonLinear)
