"""CUDA-graph capture keyed by input shape and precision configuration.

Drop-in for the reference's ``GraphReplay`` (actune/graph.py:6-95): same
constructor ``GraphReplay(function, layers, *, shared_a8=False, max_graphs=12)``,
the same ``enabled`` switch, ``replays`` / ``fallbacks`` counters and caching
contract:

* a call is identified by the argument pytree, every tensor leaf's shape, stride,
  dtype and device (non-tensor leaves by type and repr), and the active mode of
  every bank layer under the current precision profile;
* a new identity is warmed up twice on a side stream and then captured, until
  ``max_graphs`` graphs exist; beyond that the call runs eagerly and counts a
  fallback (no eviction);
* replays feed the captured per-layer ``calls`` / ``input_elements`` increments
  back into the layers (capture itself leaves the counters as they were), so
  ``BankRuntime.audit`` sees every request;
* small CUDA tensors built from Python literals inside the function
  (``torch.tensor(1.0, device="cuda")`` and the like, as OpenPI's sampler does)
  are created once while warming up and handed out as fresh clones afterwards, so
  capture issues no host-to-device copy; a literal first seen during capture is
  an error.

How it is organised here: calls are grouped by input signature into *slots*.  A
slot owns one set of static input buffers, shared by every precision
configuration captured for that signature, so switching q00/q01/q11/q10 between
calls copies the inputs into the same buffers and replays another graph -- no
per-configuration input copies.  Literal constants are intercepted with a
``TorchFunctionMode`` while warming up and capturing.  With ``shared_a8`` the
sibling projections of a captured function share one activation quantization
(the shared activation scope of kernels.grouped and the tokenwise A8/A4 cache).
"""
from __future__ import annotations

from contextlib import ExitStack, contextmanager
from dataclasses import dataclass, field
from typing import Any

import torch
from torch.overrides import TorchFunctionMode
from torch.utils import _pytree as pytree

from .kernels._tokenwise import shared_a8_cache_scope
from .kernels.grouped import shared_activation_scope
from .precision import active_precision_profile


def _is_literal(value) -> bool:
    if isinstance(value, (bool, int, float)):
        return True
    return isinstance(value, (list, tuple)) and all(_is_literal(v) for v in value)


class _LiteralConstants(TorchFunctionMode):
    """Serves CUDA ``torch.tensor(<python literal>, ...)`` calls from a cache.

    While ``capturing`` is False a new literal is materialised and remembered;
    during capture a literal not seen before raises.  Every call returns a clone,
    because callers may update such a tensor in place (a time step, say)."""

    def __init__(self, cache: dict):
        super().__init__()
        self.cache = cache
        self.capturing = False

    def __torch_function__(self, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        if func is torch.tensor and args and len(args) == 1:
            device = kwargs.get("device")
            if (device is not None and torch.device(device).type == "cuda" and _is_literal(args[0])
                    and not kwargs.get("requires_grad", False)):
                key = (repr(args[0]), repr(sorted(kwargs.items())))
                value = self.cache.get(key)
                if value is None:
                    if self.capturing or torch.cuda.is_current_stream_capturing():
                        raise RuntimeError("Unwarmed CUDA constant in graph capture")
                    value = self.cache[key] = func(*args, **kwargs)
                return value.clone()
        return func(*args, **kwargs)


@dataclass
class _Capture:
    graph: torch.cuda.CUDAGraph
    output: Any
    deltas: dict          # layer name -> (calls, input_elements) added per replay


@dataclass
class _Slot:
    statics: list         # static leaves (tensors cloned once) shared by the slot's captures
    captures: dict = field(default_factory=dict)   # per-layer modes -> _Capture


class GraphReplay:
    def __init__(self, function, layers, *, shared_a8=False, max_graphs=12):
        self.function = function
        self.layers = layers
        self.shared_a8 = shared_a8
        self.max_graphs = max_graphs
        self.enabled = False
        self.replays = 0
        self.fallbacks = 0
        self.constants: dict = {}
        self._slots: dict = {}

    # ------------------------------------------------------------------ identity
    @staticmethod
    def _signature(leaves, tree):
        sig = []
        for x in leaves:
            if isinstance(x, torch.Tensor):
                sig.append((tuple(x.shape), tuple(x.stride()), str(x.dtype), str(x.device)))
            else:
                sig.append((type(x).__name__, repr(x)))
        return str(tree), tuple(sig)

    def _modes(self):
        profile = active_precision_profile()
        return tuple(m.assignments[profile or m.default_profile] for m in self.layers.values())

    def key(self, leaves, tree):
        """The identity of a call: (pytree, leaf signature, every layer's active mode)."""
        tree_s, sig = self._signature(leaves, tree)
        return tree_s, sig, self._modes()

    @property
    def graphs(self):
        """Every captured graph by its full key."""
        return {(tree_s, sig, modes): c for (tree_s, sig), slot in self._slots.items()
                for modes, c in slot.captures.items()}

    # ------------------------------------------------------------------ scopes
    @contextmanager
    def scope(self, capturing=False):
        """Literal-constant interception plus, with shared_a8, the shared activation
        scopes; active while warming up and capturing."""
        mode = _LiteralConstants(self.constants)
        mode.capturing = capturing
        with ExitStack() as stack:
            stack.enter_context(shared_activation_scope(self.shared_a8))
            stack.enter_context(shared_a8_cache_scope(enabled=self.shared_a8))
            stack.enter_context(mode)
            yield

    # ------------------------------------------------------------------ call
    def __call__(self, *args, **kwargs):
        if not self.enabled:
            return self.function(*args, **kwargs)
        leaves, tree = pytree.tree_flatten((args, kwargs))
        slot_key = self._signature(leaves, tree)
        modes = self._modes()
        slot = self._slots.get(slot_key)
        capture = None if slot is None else slot.captures.get(modes)
        if capture is None:
            if sum(len(s.captures) for s in self._slots.values()) >= self.max_graphs:
                self.fallbacks += 1
                return self.function(*args, **kwargs)
            if slot is None:
                slot = _Slot([x.clone() if isinstance(x, torch.Tensor) else x for x in leaves])
                self._slots[slot_key] = slot
            capture = slot.captures[modes] = self._record(slot, tree)
        for src, dst in zip(leaves, slot.statics, strict=True):
            if isinstance(src, torch.Tensor) and src.data_ptr() != dst.data_ptr():
                dst.copy_(src)
        capture.graph.replay()
        for name, (calls, elements) in capture.deltas.items():
            layer = self.layers[name]
            layer.calls += calls
            layer.input_elements += elements
        self.replays += 1
        return capture.output

    def _record(self, slot, tree):
        before = {n: (m.calls, m.input_elements) for n, m in self.layers.items()}
        s_args, s_kwargs = pytree.tree_unflatten(slot.statics, tree)
        warm = torch.cuda.Stream()
        warm.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(warm), torch.inference_mode():
            for _ in range(2):
                with self.scope():
                    self.function(*s_args, **s_kwargs)
        torch.cuda.current_stream().wait_stream(warm)
        for m in self.layers.values():
            m.calls = m.input_elements = 0
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph), torch.inference_mode(), self.scope(capturing=True):
            output = self.function(*s_args, **s_kwargs)
        deltas = {n: (m.calls, m.input_elements) for n, m in self.layers.items()}
        for n, m in self.layers.items():
            m.calls, m.input_elements = before[n]
        return _Capture(graph, output, deltas)

    def release(self):
        """Drop every captured graph and static buffer (frees their memory)."""
        self._slots.clear()
