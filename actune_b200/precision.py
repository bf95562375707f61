"""Request-scoped precision profiles and the shared resident bank.

Drop-in for the reference's actune/precision.py:10-87 (and the configuration
names of actune/tree.py:13, the mode parser of actune/_allocation/pi05_budget.py:19-22):

* ``precision_profile(cfg)`` sets the active configuration (one of q00, q01,
  q11, q10) for the current thread / async task through a ContextVar;
  ``active_precision_profile()`` reads it (None outside any scope, in which
  case layers fall back to their default profile, q11).
* ``SharedBank`` holds, per targeted matrix, the mode each configuration uses
  and the storage bytes of each version; it audits the per-request W/A bit
  budget and the resident storage, raising ValueError with the reference's
  messages.
"""
from __future__ import annotations

import math
from contextlib import contextmanager
from contextvars import ContextVar
from dataclasses import dataclass

CONFIGURATIONS = ("q00", "q01", "q11", "q10")
MODES = frozenset(f"w{w}a{a}" for w in (2, 4, 8) for a in (2, 4, 8))

_ACTIVE = ContextVar("actune_precision_profile", default=None)


def pair(mode):
    """'w4a8' -> (4, 8); ValueError for anything outside the nine modes."""
    if not isinstance(mode, str) or mode not in MODES:
        raise ValueError(f"invalid pi05 precision: {mode}")
    return int(mode[1]), int(mode[3])


def active_precision_profile():
    return _ACTIVE.get()


@contextmanager
def precision_profile(configuration):
    if configuration not in CONFIGURATIONS:
        raise ValueError("Unknown ActTune configuration")
    token = _ACTIVE.set(configuration)
    try:
        yield
    finally:
        _ACTIVE.reset(token)


@dataclass
class SharedBank:
    configurations: dict      # configuration -> {matrix name -> mode}
    shapes: dict              # matrix name -> [out_features, in_features]
    activation_elements: dict  # matrix name -> activation elements per request
    shape_groups: list        # partition of matrix names by invocation shape
    version_bytes: dict       # matrix name -> {mode -> resident storage bytes}
    budget: str               # "w4a4" or "w4a8"
    storage_limit: int

    def _versions(self, name):
        return {assignment[name] for assignment in self.configurations.values()}

    def resident_bytes(self):
        return sum(self.version_bytes[name][mode] for name in self.shapes for mode in self._versions(name))

    def metrics(self, configuration, activation_elements=None):
        assignment = self.configurations[configuration]
        counts = self.activation_elements if activation_elements is None else activation_elements
        if set(counts) != set(self.shapes) or any(type(v) is not int or v <= 0 for v in counts.values()):
            raise ValueError("Every target must execute with a positive activation-element count")
        params = {name: math.prod(shape) for name, shape in self.shapes.items()}
        weight_bits = sum(params[n] * pair(m)[0] for n, m in assignment.items()) / sum(params.values())
        act_bits = sum(counts[n] * pair(m)[1] for n, m in assignment.items()) / sum(counts.values())
        group_bits = [sum(counts[n] * pair(assignment[n])[1] for n in group) / sum(counts[n] for n in group)
                      for group in self.shape_groups]
        return dict(weight_bits=weight_bits, activation_bits=act_bits, group_activation_bits=group_bits)

    def check_request(self, configuration, counts=None):
        m = self.metrics(configuration, counts)
        if m["weight_bits"] > 4 + 1e-12:
            raise ValueError("Active weight budget exceeds four bits")
        if self.budget == "w4a4" and max(m["activation_bits"], *m["group_activation_bits"]) > 4 + 1e-12:
            raise ValueError("Active activation budget exceeds four bits")
        if self.budget == "w4a8" and any(pair(v)[1] != 8 for v in self.configurations[configuration].values()):
            raise ValueError("W4A8 requires A8 on every target")
        return m

    def validate(self):
        if self.budget not in ("w4a4", "w4a8") or set(self.configurations) != set(CONFIGURATIONS):
            raise ValueError("Expected a W4A4/W4A8 bank with four configurations")
        if not self.shapes or any(len(s) != 2 or any(type(v) is not int or v <= 0 for v in s)
                                  for s in self.shapes.values()):
            raise ValueError("Invalid matrix shapes")
        flat = sorted(n for group in self.shape_groups for n in group)
        if flat != sorted(self.shapes) or any(not group for group in self.shape_groups):
            raise ValueError("Invocation-shape groups must partition the targeted layers")
        if any(set(assignment) != set(self.shapes) for assignment in self.configurations.values()):
            raise ValueError("Configuration coverage differs from targeted layers")
        versions = {n: self._versions(n) for n in self.shapes}
        if sorted(len(v) for v in versions.values() if len(v) > 1) != [2, 2]:
            raise ValueError("Paper bank requires exactly two binary switchable matrices")
        realised = {tuple(assignment[n] for n in sorted(self.shapes)) for assignment in self.configurations.values()}
        if len(realised) != 4:
            raise ValueError("Configurations must realize all four alternatives")
        for n, modes in versions.items():
            for mode in modes:
                pair(mode)
                size = self.version_bytes[n][mode]
                if type(size) is not int or size <= 0:
                    raise ValueError("Version storage must include packed weights, scales and bias")
        for configuration in CONFIGURATIONS:
            self.check_request(configuration)
        if self.storage_limit <= 0 or self.resident_bytes() > self.storage_limit:
            raise ValueError("All resident versions together exceed storage budget")
        return self
