"""Group-64 packed W{2,4,8} x A{2,4,8} linear layers (drop-in for actune.kernels.grouped).

Same classes, constructor arguments, buffer names/shapes/dtypes and forward
contract as the reference's actune/kernels/grouped.py:

* ``GroupedLinear(linear, w, a, ratios)`` (reference :114-143): buffers
  ``packed_weight`` uint8 [N, K*w/8], ``weight_scale`` f32 [N], ``bias``
  (layer dtype, f32 when a == 4, or None).  ``forward(x)`` needs a CUDA ``x[..., K]``
  and returns ``[..., N]`` in ``x.dtype``.
* ``GroupedPaddedLinear(linear, assignments, initial, clips)`` (reference
  :146-167): K zero-padded to a multiple of 128, one backend per distinct mode,
  backend chosen by the request's precision profile (fallback ``initial``),
  ``calls``/``input_elements`` counters.
* ``pack_rows``, ``extension().linear(...)``, ``reuse_mlp_temporary``.

The two launches of the reference forward (Triton quantizer, then the
mma.sync / Triton GEMM) become two sm_100a kernels behind the C ABI:
``actune_quantize_group64`` and ``actune_packed_linear`` (tcgen05 kind::i8).
"""
from __future__ import annotations

from contextlib import contextmanager
from contextvars import ContextVar
from types import MethodType

import torch

from .. import _lib, ops
from ..precision import active_precision_profile
from .quantizers import weight_codes


# Sibling projections (Q/K/V, gate/up) read the same input.  Inside
# shared_activation_scope(True) the packed activations of the most recent
# inputs are kept and reused when the same tensor (same storage, version,
# shape, dtype) is quantized again to the same width.  The cached entry holds a
# reference to the input, so its memory cannot be recycled while cached.
_SHARED = ContextVar("actune_shared_activation_cache", default=None)
_SHARED_CAPACITY = 4


@contextmanager
def shared_activation_scope(enabled=True):
    token = _SHARED.set([] if enabled else None)
    try:
        yield
    finally:
        _SHARED.reset(token)


def _version(t):
    # Inference-mode tensors carry no version counter: within one scope they are
    # matched by storage, shape, dtype and width alone (an in-place update of such
    # an input between two projections of the same scope is not detected).
    return -1 if t.is_inference() else t._version


def shared_activation_active():
    """True inside an enabled shared_activation_scope."""
    return _SHARED.get() is not None


def share_quantized(flat, bits, packed, scales, codes8=False):
    """Offer already quantized activations of `flat` (bit-identical to what
    ``ops.quantize_group64(flat, bits, codes8=codes8)`` returns) to the active shared
    activation scope, so the next projection reading `flat` reuses them.  No-op
    outside one."""
    cache = _SHARED.get()
    if cache is None:
        return False
    key = (flat.data_ptr(), _version(flat), tuple(flat.shape), flat.dtype, flat.device, bits, bool(codes8))
    cache.append((key, flat, packed, scales))
    if len(cache) > _SHARED_CAPACITY:
        cache.pop(0)
    return True


def _quantize_shared(flat, bits, codes8=False):
    cache = _SHARED.get()
    if cache is None:
        return ops.quantize_group64(flat, bits, codes8=codes8)
    key = (flat.data_ptr(), _version(flat), tuple(flat.shape), flat.dtype, flat.device, bits, bool(codes8))
    for entry_key, _, packed, scales in cache:
        if entry_key == key:
            return packed, scales
    packed, scales = ops.quantize_group64(flat, bits, codes8=codes8)
    cache.append((key, flat, packed, scales))
    if len(cache) > _SHARED_CAPACITY:
        cache.pop(0)
    return packed, scales


def _inference_mlp(self, x):
    if torch.is_grad_enabled():
        return self._group64_original_forward(x)
    # Reuse the gate activation buffer for the product: two intermediate-width
    # tensors live instead of three (reference grouped.py:18-25).
    gate = self.act_fn(self.gate_proj(x))
    gate.mul_(self.up_proj(x))
    return self.down_proj(gate)


def reuse_mlp_temporary(model):
    """Patch every Gemma MLP of ``model`` to reuse its gate temporary; returns the count."""
    from transformers.models.gemma.modeling_gemma import GemmaMLP
    patched = 0
    for module in model.modules():
        if type(module) is GemmaMLP and not hasattr(module, "_group64_original_forward"):
            module._group64_original_forward = module.forward
            module.forward = MethodType(_inference_mlp, module)
            patched += 1
    return patched


def unpack_rows(packed, bits, k):
    """Inverse of ``pack_rows``: int8 codes [R, k] from little-endian packed rows
    (code j of a row sits in bits [bits*(j % per_byte), ...) of byte j // per_byte,
    two's complement).  Install-time helper, runs where ``packed`` lives."""
    if bits == 8:
        return packed.view(torch.int8)[:, :k].contiguous()
    per = 8 // bits
    p = packed.view(torch.int8)
    parts = [torch.bitwise_right_shift(torch.bitwise_left_shift(p, 8 - bits * (j + 1)), 8 - bits)
             for j in range(per)]
    return torch.stack(parts, dim=-1).reshape(p.shape[0], -1)[:, :k].contiguous()


def pack_rows(q, bits):
    """Little-endian sub-byte packing of int8 codes [R, K] (reference grouped.py:108-111).

    Runs on the GPU; a CPU tensor is packed on the current CUDA device and the
    result returned on the input's device."""
    src = q if q.is_cuda else q.to("cuda")
    out = ops.pack_rows(src.to(torch.int8).contiguous(), bits)
    return out.to(q.device)


class _Extension:
    """The reference's native-op surface: ``extension().linear(a, as, w, ws, bias, source, W, A[, config])``."""

    @staticmethod
    def linear(a, as_, w, ws, bias, source, W, A, config=None):
        if not (a.is_cuda and as_.is_cuda and w.is_cuda and ws.is_cuda and bias.is_cuda and source.is_cuda):
            raise RuntimeError("CUDA required")
        if source.dim() != 2:
            raise RuntimeError("rank mismatch")
        m, k = source.shape
        variant = _lib.VARIANT_AUTO if config is None else int(config)
        if variant < 0 or variant > _lib.VARIANT_MAX:
            raise RuntimeError("invalid configuration")
        with torch.cuda.device(source.device):
            return ops.packed_linear(a, as_, w, ws, None if bias.numel() == 0 else bias, k, int(W), int(A),
                                     out_dtype=source.dtype, variant=variant)


_EXTENSION = _Extension()


def extension():
    """The loaded C-ABI library as the reference's extension object (loads it, raises if missing)."""
    _lib.lib()
    return _EXTENSION


# The weight-streaming kernel (up to 32 token rows) is bound by reading the packed
# weights, so it keeps them packed; the tile kernel above that is not, and runs
# faster on int8 codes (no per-tile expansion of sub-byte codes).
DECODED_MIN_TOKENS = 33


class GroupedLinear(torch.nn.Module):
    """``decode_weight()`` keeps, next to the packed rows, the weight codes as int8
    bytes [N, K] (the W=8 packed form; not a buffer: the bank's storage audit counts
    the packed versions only).  Calls with more than 32 token rows then quantize
    their activations to the same A-bit codes written one byte each and run the
    W=8 / A=8 kernel: the integer group dots and the scales are the same numbers,
    so outputs are bit-identical, for N*K extra bytes of device memory."""

    def __init__(self, linear, w, a, ratios):
        super().__init__()
        self.in_features = linear.in_features
        self.out_features = linear.out_features
        self.w, self.a = w, a
        if self.in_features % 64:
            raise ValueError("Grouped backend requires K divisible by 64")
        if w not in (2, 4, 8) or a not in (2, 4, 8):
            raise ValueError("Unsupported integer width")
        codes, scale = weight_codes(linear.weight, w, a, clip_ratios=ratios)
        self.register_buffer("packed_weight", pack_rows(codes, w))
        self.register_buffer("weight_scale", scale.contiguous())
        bias = None if linear.bias is None else linear.bias.detach().clone()
        if bias is not None and a == 4:
            bias = bias.float()
        self.register_buffer("bias", bias)
        self.variant = _lib.VARIANT_AUTO
        self.decoded_weight = None

    def decode_weight(self):
        """Keep the int8 weight codes for calls of more than 32 token rows (W < 8);
        returns the bytes added.  The decoded rows are checked to pack back to the
        stored ones."""
        if self.w == 8 or self.decoded_weight is not None:
            return 0
        codes = unpack_rows(self.packed_weight, self.w, self.in_features)
        if not torch.equal(ops.pack_rows(codes, self.w), self.packed_weight):
            raise RuntimeError("decoded weight codes do not pack back to the stored rows")
        self.decoded_weight = codes.view(torch.uint8)  # the W=8 packed form: one byte per code
        return codes.numel()

    def decoded_path(self, rows):
        """True when a call of `rows` token rows runs on the decoded codes."""
        return self.decoded_weight is not None and rows >= DECODED_MIN_TOKENS

    def activation_format(self, rows):
        """(bits, codes8): the quantization of a call's activations (``codes8``: the
        A-bit codes one byte each)."""
        return self.a, self.decoded_path(rows) and self.a < 8

    def operands(self, rows):
        """(weight, W, A) the kernel of a call of `rows` token rows runs with."""
        if self.decoded_path(rows):
            return self.decoded_weight, 8, 8
        return self.packed_weight, self.w, self.a

    def forward(self, x):
        if not x.is_cuda:
            raise ValueError("Grouped integer backend requires CUDA")
        flat = x.reshape(-1, self.in_features).contiguous()
        rows = flat.shape[0]
        acts, scales = _quantize_shared(flat, *self.activation_format(rows))
        weight, w, a = self.operands(rows)
        out = ops.packed_linear(acts, scales, weight, self.weight_scale, self.bias,
                                self.in_features, w, a, out_dtype=x.dtype, variant=self.variant)
        return out.reshape(*x.shape[:-1], self.out_features)


def decode_weights(model):
    """``decode_weight()`` on every GroupedLinear of ``model``; returns the bytes added."""
    return sum(m.decode_weight() for m in model.modules() if isinstance(m, GroupedLinear))


class GroupedPaddedLinear(torch.nn.Module):
    def __init__(self, linear, assignments, initial, clips):
        super().__init__()
        logical = linear.in_features
        padded = (logical + 127) // 128 * 128
        if padded != logical:
            wide = torch.nn.Linear(padded, linear.out_features, bias=linear.bias is not None,
                                   device=linear.weight.device, dtype=linear.weight.dtype)
            with torch.no_grad():
                wide.weight.zero_()
                wide.weight[:, :logical].copy_(linear.weight)
                if wide.bias is not None:
                    wide.bias.copy_(linear.bias)
            linear = wide
        self.in_features = logical
        self.out_features = linear.out_features
        self.padding = padded - logical
        self.assignments = dict(assignments)
        self.default_profile = initial
        modes = sorted(set(self.assignments.values()))
        self.backends = torch.nn.ModuleDict(
            {mode: GroupedLinear(linear, int(mode[1]), int(mode[3]), clips[mode]) for mode in modes})
        self.register_buffer("_weight_dtype", torch.empty(0, device=linear.weight.device, dtype=linear.weight.dtype))
        self.calls = 0
        self.input_elements = 0

    @property
    def weight(self):
        return self._weight_dtype

    def active_backend(self):
        return self.backends[self.assignments[active_precision_profile() or self.default_profile]]

    def forward(self, x):
        self.calls += 1
        self.input_elements += x.numel()
        if self.padding:
            x = torch.nn.functional.pad(x, (0, self.padding))
        return self.active_backend()(x)
