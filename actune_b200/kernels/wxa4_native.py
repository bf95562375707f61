"""Per-row A4 backends: drop-in for the reference's actune/kernels/wxa4_native.py.

Same public surface: ``W2A4NativeLinear`` / ``W4A4NativeLinear`` (``linear``,
``weight_clip_ratios``) with buffers ``packed_weight`` u8 [N, K*W/8] (row-major,
consecutive codes of a row packed little-endian, wxa4_native.py:200-214),
``weight_scale`` f32 [N] and ``bias`` f32 [N] (empty when the Linear has none);
``W8A4NativeLinear`` with ``weight_int8`` int8 [K, N] holding the nested code
16*q4 + r4 and ``weight_scale`` = the W4 scale / 16 (wxa4_native.py:313-338).

Activations: one dynamic INT4 scale per row, ``max(absmax, 1e-8) * fp32(1/7)``,
packed two codes per byte (``ops.quantize_rows_a4``), shared by sibling
projections inside ``shared_a8_cache_scope``.  W8A4 consumes the same packed rows
(the reference widens them to an INT8 copy first).

GEMM: ``ops.rowwise_linear`` -- exact INT32 dots over all of K on the tcgen05
INT8 tensor cores (sub-byte codes widened in shared memory; Blackwell has no
INT4 MMA), then the reference's epilogue bit for bit: ``float(acc) * (as * ws)
(+ bias)`` for W{2,4}A4 (the native S4 kernel, native_s4_extension_kernel.cu:
226-234) and ``(float(acc) * as) * ws (+ bias)`` for W8A4 (the W8A8 Triton
kernel it runs, wxa4_native.py:370-389).  Decode sizes (M <= 16) stream the
weights through the weight-streaming kernel instead.
"""
from __future__ import annotations

import torch

from .. import ops
from ._tokenwise import quantize_rows_a4_shared as _quantize_a4_shared
from .quantizers import signed_r4_refine, symmetric_int2_quantize, symmetric_int4_quantize

COMPUTE_INSTRUCTION = "tcgen05.mma.kind::i8 (sub-byte codes widened to S8 in shared memory)"


def _pack_signed(values: torch.Tensor, bits: int) -> torch.Tensor:
    """Pack consecutive signed codes along K, keeping row-major weights."""
    if bits not in (2, 4):
        raise ValueError("bits must be 2 or 4")
    if values.is_cuda:
        return ops.pack_rows(values.to(torch.int8).contiguous(), bits)
    per = 8 // bits
    v = (values.to(torch.int16) & ((1 << bits) - 1)).reshape(values.shape[0], -1, per)
    out = torch.zeros(v.shape[:2], dtype=torch.int16)
    for i in range(per):
        out |= v[..., i] << (i * bits)
    return out.to(torch.uint8).contiguous()


def _bias_buffer(linear: torch.nn.Linear) -> torch.Tensor:
    if linear.bias is None:
        return torch.empty(0, dtype=torch.float32, device=linear.weight.device)
    return linear.bias.detach().float().contiguous()


def _check_input(value: torch.Tensor, what: str) -> None:
    if not value.is_cuda:
        raise ValueError(f"{what} requires a CUDA input")
    major, _minor = torch.cuda.get_device_capability(value.device)
    if major != 10:
        raise RuntimeError(f"{what} requires a compute capability 10.x (B200) device")


class _WxA4NativeLinear(torch.nn.Module):
    weight_bits: int

    def __init__(self, linear: torch.nn.Linear, *, weight_bits: int, weight_clip_ratios=None) -> None:
        super().__init__()
        if linear.in_features % 64:
            raise ValueError("native S4 MMA requires in_features divisible by 64")
        if weight_bits not in (2, 4):
            raise ValueError("weight_bits must be 2 or 4")
        self.in_features = linear.in_features
        self.out_features = linear.out_features
        self.weight_bits = weight_bits
        with torch.no_grad():
            quantize = symmetric_int2_quantize if weight_bits == 2 else symmetric_int4_quantize
            quantized, scale = quantize(linear.weight, clip_ratios=weight_clip_ratios)
            packed = _pack_signed(quantized, weight_bits)
        self.register_buffer("packed_weight", packed)
        self.register_buffer("weight_scale", scale.contiguous())
        self.register_buffer("bias", _bias_buffer(linear))
        self.weight_quantizer = (f"rtn_per_output_row_w{weight_bits}_v1" if weight_clip_ratios is None
                                 else "awq_style_joint_precision_lattice_clip_v1")
        self.activation_quantizer = "dynamic_per_row_s4_v1"
        self.compute_instruction = COMPUTE_INSTRUCTION
        self.native_int4_tensor_core = False
        self.native_int8_tensor_core = True

    def forward(self, value: torch.Tensor) -> torch.Tensor:
        _check_input(value, "native S4 MMA")
        original_shape = value.shape[:-1]
        flat = value.reshape(-1, self.in_features)
        packed, activation_scale = _quantize_a4_shared(value, flat, in_features=self.in_features)
        output = ops.rowwise_linear(packed, 4, activation_scale, self.packed_weight, self.weight_bits,
                                    self.weight_scale, self.bias, self.in_features, order=ops.ORDER_NATIVE,
                                    out_dtype=value.dtype)
        return output.reshape(*original_shape, self.out_features)


class W2A4NativeLinear(_WxA4NativeLinear):
    def __init__(self, linear: torch.nn.Linear, *, weight_clip_ratios=None) -> None:
        super().__init__(linear, weight_bits=2, weight_clip_ratios=weight_clip_ratios)


class W4A4NativeLinear(_WxA4NativeLinear):
    def __init__(self, linear: torch.nn.Linear, *, weight_clip_ratios=None) -> None:
        super().__init__(linear, weight_bits=4, weight_clip_ratios=weight_clip_ratios)


class W8A4NativeLinear(torch.nn.Module):
    """INT8-weight / A4 Linear: one INT8 tensor-core GEMM on the packed A4 rows."""

    def __init__(self, linear: torch.nn.Linear, *, weight_clip_ratios=None) -> None:
        super().__init__()
        if linear.in_features % 128:
            raise ValueError("W8A4 S8 MMA requires in_features divisible by 128")
        self.in_features = linear.in_features
        self.out_features = linear.out_features
        with torch.no_grad():
            q4, scale4 = symmetric_int4_quantize(linear.weight, clip_ratios=weight_clip_ratios)
            _residual, q8 = signed_r4_refine(linear.weight, q4, scale4)
        self.register_buffer("weight_int8", q8.t().contiguous())
        self.register_buffer("weight_scale", (scale4 / 16.0).contiguous())
        self.register_buffer("bias", _bias_buffer(linear))
        # The kernel reads the codes as rows [N, K]; rebuilt from weight_int8 on load.
        self.register_buffer("_rows", q8.to(torch.int8).contiguous().view(torch.uint8), persistent=False)
        self.register_load_state_dict_post_hook(lambda module, _keys: module._refresh_rows())
        self.weight_bits = 8
        self.weight_quantizer = ("nested_signed_w8_rtn_v1" if weight_clip_ratios is None
                                 else "awq_style_joint_precision_lattice_clip_v1")
        self.activation_quantizer = "dynamic_per_row_s4_v1"
        self.compute_instruction = COMPUTE_INSTRUCTION
        self.native_int4_tensor_core = False
        self.native_int8_tensor_core = True
        self.a4_sign_extended_to_int8 = True
        self.s4_mma_count_per_k_tile = 0

    def _refresh_rows(self):
        self._rows = self.weight_int8.t().contiguous().view(torch.uint8)

    def forward(self, value: torch.Tensor) -> torch.Tensor:
        _check_input(value, "W8A4 integer MMA")
        original_shape = value.shape[:-1]
        flat = value.reshape(-1, self.in_features)
        packed, activation_scale = _quantize_a4_shared(value, flat, in_features=self.in_features)
        if self._rows.device != flat.device:
            self._rows = self._rows.to(flat.device)
        output = ops.rowwise_linear(packed, 4, activation_scale, self._rows, 8, self.weight_scale, self.bias,
                                    self.in_features, order=ops.ORDER_TRITON, out_dtype=value.dtype)
        return output.reshape(*original_shape, self.out_features)

