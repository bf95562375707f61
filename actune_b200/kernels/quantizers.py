"""Install-time weight codebooks on the GPU.

Same functions, arguments, return values and ValueError messages as the
reference's actune/kernels/quantizers.py:4-94; the arithmetic runs in
``weight_codes_kernel`` (csrc/quantize.cu) through the C ABI:

* W4:          scale = max(row absmax, 1e-8) * clip / 7,  codes in [-8, 7]
* W2:          scale = max(row absmax, 1e-8) * clip,      codes in [-2, 1]
* W8, A != 4:  scale = max(row absmax, 1e-8) / 127 (clip ignored), codes in [-128, 127]
* W8, A == 4:  nested code 16*q4 + r4 with the W4 scale / 16

A CPU weight is quantized on the current CUDA device and the results are
returned on the weight's device (there is no CPU implementation).
"""
from __future__ import annotations

import torch

from .. import ops


def _validate_clip_ratios(clip_ratios, *, out_features: int, device) -> torch.Tensor:
    ratio = torch.as_tensor(clip_ratios, dtype=torch.float32, device=device).flatten()
    if ratio.numel() == 1:
        ratio = ratio.expand(out_features)
    if ratio.numel() != out_features:
        raise ValueError(f"expected {out_features} AWQ-style clip ratios, got {ratio.numel()}")
    if not torch.isfinite(ratio).all():
        raise ValueError("AWQ-style clip ratios must be finite")
    if bool(((ratio <= 0.0) | (ratio > 1.0)).any()):
        raise ValueError("AWQ-style clip ratios must lie in (0, 1]")
    return ratio.contiguous()


def _on_gpu(weight: torch.Tensor) -> torch.Tensor:
    w = weight.detach()
    if not w.is_cuda:
        if not torch.cuda.is_available():
            raise RuntimeError("weight quantization runs on the GPU; no CUDA device is available")
        w = w.to("cuda")
    if w.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        w = w.float()
    return w.contiguous()


def _codes(weight, w_bits, a_bits, clip_ratios):
    w = _on_gpu(weight)
    clip = None
    if clip_ratios is not None:
        clip = _validate_clip_ratios(clip_ratios, out_features=w.shape[0], device=w.device)
    q, s = ops.weight_codes(w, w_bits, a_bits, clip)
    return q.to(weight.device), s.to(weight.device)


def symmetric_int4_quantize(weight, *, clip_ratios=None):
    """Signed INT4 rows: (codes int8 in [-8, 7], per-row scale)."""
    return _codes(weight, 4, 8, clip_ratios)


def symmetric_int2_quantize(weight, *, clip_ratios=None):
    """Signed INT2 rows: (codes int8 in [-2, 1], per-row scale = clipped absmax)."""
    return _codes(weight, 2, 8, clip_ratios)


def signed_r4_refine(weight, q4, scale4):
    """Signed R4 residual and the nested INT8 code 16*q4 + r4 (reference quantizers.py:42-57)."""
    w = _on_gpu(weight)
    residual, q8 = ops.r4_refine(w, q4, scale4)
    return residual.to(weight.device), q8.to(weight.device)


def weight_codes(weight, w, a, *, clip_ratios=None):
    """Codes and per-row scale of the W{2,4,8} codebook used with activation width ``a``."""
    if w not in (2, 4, 8) or a not in (2, 4, 8):
        raise ValueError("Unsupported integer width")
    return _codes(weight, w, a, clip_ratios)
