"""Shape- and precision-keyed CUDA Graph replay (drop-in for the reference's actune/graph.py:6-95).

``GraphReplay(function, layers, *, shared_a8=False, max_graphs=12)`` wraps a
forward function.  While ``enabled`` is False it just calls the function.  Once
enabled, each call is keyed by (argument pytree, every tensor's shape / stride /
dtype / device, the active mode of every layer under the current precision
profile); a new key (while fewer than ``max_graphs`` exist) is warmed twice on
a side stream and captured, later calls copy their inputs into the captured
static inputs and replay.  Switching q00/q01/q11/q10 therefore selects another
captured graph instead of re-launching kernels.  Per-layer ``calls`` /
``input_elements`` counters are restored after capture and advanced by the
captured amounts on every replay, so ``BankRuntime.audit`` still sees them.

``scope()`` is active during warm-up and capture: it pre-creates small CUDA
constants built from Python literals with ``torch.tensor`` (so capture issues no
host->device copy) and, with ``shared_a8=True``, lets sibling projections that
read the same input share one quantization (``shared_activation_scope``).
"""
from __future__ import annotations

from contextlib import contextmanager
from unittest.mock import patch

import torch

from .kernels._tokenwise import shared_a8_cache_scope
from .kernels.grouped import shared_activation_scope
from .precision import active_precision_profile


class GraphReplay:
    def __init__(self, function, layers, *, shared_a8=False, max_graphs=12):
        self.function = function
        self.layers = layers
        self.shared_a8 = shared_a8
        self.max_graphs = max_graphs
        self.graphs = {}
        self.enabled = False
        self.replays = 0
        self.fallbacks = 0
        self.constants = {}

    @contextmanager
    def scope(self):
        original = torch.tensor

        def is_literal(value):
            if isinstance(value, (bool, int, float)):
                return True
            return isinstance(value, (list, tuple)) and all(is_literal(v) for v in value)

        def constant(data, *args, **kwargs):
            device = kwargs.get("device")
            if device is None or torch.device(device).type != "cuda":
                return original(data, *args, **kwargs)
            if not is_literal(data) or args or kwargs.get("requires_grad", False):
                return original(data, *args, **kwargs)
            key = (repr(data), repr(sorted(kwargs.items())))
            if key not in self.constants:
                if torch.cuda.is_current_stream_capturing():
                    raise RuntimeError("Unwarmed CUDA constant in graph capture")
                self.constants[key] = original(data, **kwargs)
            # Clone: callers may update such constants in place (e.g. a time step).
            return self.constants[key].clone()

        with shared_activation_scope(self.shared_a8), shared_a8_cache_scope(enabled=self.shared_a8), \
                patch.object(torch, "tensor", constant):
            yield

    def key(self, leaves, tree):
        signature = tuple((tuple(x.shape), tuple(x.stride()), str(x.dtype), str(x.device))
                          if isinstance(x, torch.Tensor) else (type(x).__name__, repr(x)) for x in leaves)
        profile = active_precision_profile()
        modes = tuple(m.assignments[profile or m.default_profile] for m in self.layers.values())
        return (str(tree), signature, modes)

    def __call__(self, *args, **kwargs):
        if not self.enabled:
            return self.function(*args, **kwargs)
        from torch.utils import _pytree as pytree
        leaves, tree = pytree.tree_flatten((args, kwargs))
        key = self.key(leaves, tree)
        if key not in self.graphs:
            if len(self.graphs) >= self.max_graphs:
                self.fallbacks += 1
                return self.function(*args, **kwargs)
            self.graphs[key] = self._capture(leaves, tree)
        graph, static, output, counts = self.graphs[key]
        for src, dst in zip(leaves, static, strict=True):
            if isinstance(src, torch.Tensor):
                dst.copy_(src)
        graph.replay()
        for name, (calls, elements) in counts.items():
            self.layers[name].calls += calls
            self.layers[name].input_elements += elements
        self.replays += 1
        return output

    def _capture(self, leaves, tree):
        from torch.utils import _pytree as pytree
        saved = {n: (m.calls, m.input_elements) for n, m in self.layers.items()}
        static = [x.clone() if isinstance(x, torch.Tensor) else x for x in leaves]
        static_args, static_kwargs = pytree.tree_unflatten(static, tree)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side), torch.inference_mode():
            for _ in range(2):
                with self.scope():
                    self.function(*static_args, **static_kwargs)
        torch.cuda.current_stream().wait_stream(side)
        for m in self.layers.values():
            m.calls = m.input_elements = 0
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph), torch.inference_mode(), self.scope():
            output = self.function(*static_args, **static_kwargs)
        counts = {n: (m.calls, m.input_elements) for n, m in self.layers.items()}
        for n, m in self.layers.items():
            m.calls, m.input_elements = saved[n]
        return graph, static, output, counts

    def release(self):
        """Drop every captured graph (frees their memory pools)."""
        self.graphs.clear()
