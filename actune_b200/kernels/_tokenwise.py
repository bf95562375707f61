"""Shared machinery of the tokenwise W{4,8,2}A8 backends.

The reference's tokenwise modules (actune/kernels/w4a8_triton.py, w8a8_triton.py,
w2a8_triton.py) quantize each input row to INT8 with one scale per row, multiply
by per-output-channel integer weights with an exact INT32 accumulation over all
of K, and apply ``float(acc) * row_scale * weight_scale (+ bias)``.  Here that is
``ops.quantize_rows_a8`` and ``ops.tokenwise_linear`` (the tcgen05 GEMM with one
full-K accumulator per tile).

Weights: each module keeps the reference's buffer (K-major ``packed_weight`` or
``weight_int8``, so state dicts and byte counts carry over) and, as a
non-persistent buffer, the same codes packed as rows [N, K*W/8] for the kernel
(rebuilt whenever a state dict is loaded).

Sibling projections: ``shared_a8_cache_scope`` keeps the quantized activations of
the most recent input so Q/K/V and gate/up reuse one quantization
(w4a8_triton.py:204-325); the per-row A4 backends keep theirs in the same scope's
``a4_entry`` (wxa4_native.py:123-160).
"""
from __future__ import annotations

from contextlib import contextmanager
from contextvars import ContextVar
from typing import Iterator

import torch

from .. import ops


class _SharedA8Entry:
    """One task-local dynamic-A8 result shared by sibling projections."""

    __slots__ = ("source", "in_features", "activation", "scale")

    def __init__(self, source, in_features, activation, scale):
        self.source = source
        self.in_features = in_features
        self.activation = activation
        self.scale = scale


class SharedA8CacheStats:
    """Statistics and the one-entry workspace of a shared A8 scope."""

    __slots__ = ("enabled", "entry", "a4_entry", "hits", "misses")

    def __init__(self, *, enabled: bool = True) -> None:
        self.enabled = enabled
        self.entry = None
        self.a4_entry = None
        self.hits = 0
        self.misses = 0


_SHARED_A8_STATE: ContextVar[SharedA8CacheStats | None] = ContextVar(
    "actune_b200_shared_dynamic_a8_state", default=None)


def clear_shared_a8_cache() -> None:
    """Drop the task-local sibling-projection activation cache."""
    state = _SHARED_A8_STATE.get()
    if state is None:
        _SHARED_A8_STATE.set(SharedA8CacheStats())
    else:
        state.entry = None
        state.a4_entry = None


@contextmanager
def shared_a8_cache_scope(*, enabled: bool = True) -> Iterator[SharedA8CacheStats]:
    """Bound the cache's lifetime to one policy forward and release its workspace."""
    state = SharedA8CacheStats(enabled=enabled)
    token = _SHARED_A8_STATE.set(state)
    try:
        yield state
    finally:
        _SHARED_A8_STATE.reset(token)


def quantize_rows_shared(source: torch.Tensor, flat: torch.Tensor, *, in_features: int):
    """Per-row INT8 activations of ``flat``, reused for the next projection reading
    the same ``source`` object with the same K (w4a8_triton.py:262-325)."""
    if not source.is_cuda or flat.shape[-1] != in_features:
        raise ValueError("shared A8 quantization requires a CUDA input with matching K")
    state = _SHARED_A8_STATE.get()
    if state is None:
        state = SharedA8CacheStats()
        _SHARED_A8_STATE.set(state)
    entry = state.entry
    if (state.enabled and entry is not None and entry.source is source and entry.in_features == in_features
            and entry.activation.shape == flat.shape):
        state.hits += 1
        return entry.activation, entry.scale
    activation, scale = ops.quantize_rows_a8(flat.contiguous())
    state.misses += 1
    state.entry = _SharedA8Entry(source, in_features, activation, scale) if state.enabled else None
    return activation, scale


class _SharedA4Entry:
    """One task-local dynamic-A4 result (packed nibble rows and row scales)."""

    __slots__ = ("source", "in_features", "packed", "scale")

    def __init__(self, source, in_features, packed, scale):
        self.source = source
        self.in_features = in_features
        self.packed = packed
        self.scale = scale


def quantize_rows_a4_shared(source: torch.Tensor, flat: torch.Tensor, *, in_features: int):
    """Per-row INT4 activations of ``flat`` as packed nibble rows [M, K/2] and row
    scales, reused by the next A4 projection reading the same ``source`` object
    inside a ``shared_a8_cache_scope``; outside a scope nothing is cached
    (wxa4_native.py:123-160)."""
    if not source.is_cuda or flat.shape[-1] != in_features:
        raise ValueError("native A4 quantization requires a CUDA input with matching K")
    state = _SHARED_A8_STATE.get()
    entry = None if state is None else state.a4_entry
    if (entry is not None and entry.source is source and entry.in_features == in_features
            and entry.packed.shape[0] == flat.shape[0]):
        return entry.packed, entry.scale
    packed, scale = ops.quantize_rows_a4(flat.contiguous())
    if state is not None and state.enabled:
        state.a4_entry = _SharedA4Entry(source, in_features, packed, scale)
    return packed, scale


class TokenwiseLinear(torch.nn.Module):
    """Common forward of the W{4,8,2}A8 tokenwise modules."""

    bits = 8

    def _init_common(self, linear, fused_quantization, codes):
        self.in_features = linear.in_features
        self.out_features = linear.out_features
        self.fused_quantization = fused_quantization
        self.register_buffer("_rows", self._pack_rows(codes), persistent=False)
        if linear.bias is None:
            self.register_buffer("bias", None)
        else:
            self.register_buffer("bias", linear.bias.detach().clone())
        self.register_load_state_dict_post_hook(lambda module, _keys: module._refresh_rows())

    def _pack_rows(self, codes):
        """Codes [N, K] int8 -> rows [N, K*W/8] u8 (the kernel's weight layout)."""
        c = codes.to(torch.int8)
        if not c.is_cuda:
            return self._pack_rows_cpu(c)
        return ops.pack_rows(c.contiguous(), self.bits)

    def _pack_rows_cpu(self, c):
        # The same little-endian row packing on the host (install on a CPU module).
        per = 8 // self.bits
        mask = (1 << self.bits) - 1
        v = (c.to(torch.int16) & mask).reshape(c.shape[0], -1, per)
        out = torch.zeros(v.shape[:2], dtype=torch.int16)
        for i in range(per):
            out |= v[..., i] << (i * self.bits)
        return out.to(torch.uint8)

    def _codes_from_buffer(self):
        raise NotImplementedError

    def _refresh_rows(self):
        self._rows = self._pack_rows(self._codes_from_buffer()).to(self.weight_scale.device)

    def _quantize(self, flat, *, source=None):
        if self.fused_quantization:
            return quantize_rows_shared(flat if source is None else source, flat, in_features=self.in_features)
        # Eager form of the same formula (bit-identical on CUDA).
        return ops.quantize_rows_a8(flat.contiguous())

    def forward(self, value: torch.Tensor) -> torch.Tensor:
        original_shape = value.shape[:-1]
        flat = value.reshape(-1, self.in_features)
        activation, scale = self._quantize(flat, source=value)
        if self._rows.device != flat.device:
            self._rows = self._rows.to(flat.device)
        output = ops.tokenwise_linear(activation, scale, self._rows, self.weight_scale, self.bias, self.in_features,
                                      self.bits, out_dtype=value.dtype)
        return output.reshape(*original_shape, self.out_features)


def replace_with(module: torch.nn.Module, filter_fn, factory) -> int:
    replaced = 0
    for name, child in list(module.named_children()):
        if filter_fn(child, name):
            setattr(module, name, factory(child))
            replaced += 1
        else:
            replaced += replace_with(child, filter_fn, factory)
    return replaced
