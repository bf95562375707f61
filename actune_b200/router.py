"""Per-request precision routing: drop-in for the reference's PrecisionTree and
action features (actune/tree.py:102-153, actune/features.py:4-96).

Same surface: ``PrecisionTree(tree, state_dim, *, fallback="q11")`` built from the
reference's nested tree dictionaries (``profile_index`` on every node,
``feature`` / ``threshold`` / ``left`` / ``right`` on splits), ``route_vector(x)``,
``route(previous_features, state)`` returning ``Decision(region, configuration)``,
``save`` / ``load`` of the ``actune_precision_tree_v1`` JSON artefact, and
``action_forecast_features(actions, *, gripper_margin)``.  The walk and the
feature arithmetic run in C++ (include/actune_router.h); ``route_batch`` routes a
whole batch of environments in one call.
"""
from __future__ import annotations

import ctypes
import json
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from . import _lib
from .precision import CONFIGURATIONS

ACTION_FORECAST_FEATURE_NAMES = (
    "translation_energy",
    "rotation_energy",
    "translation_variation",
    "rotation_variation",
    "translation_curvature",
    "rotation_curvature",
    "translation_cancellation",
    "rotation_cancellation",
    "chunk_variation",
    "chunk_curvature",
    "cancellation",
    "gripper_transition",
    "gripper_margin",
)
MAX_STATE_DIM = 64

_DECLARED = False


def _lib_router():
    global _DECLARED
    L = _lib.lib()
    if not _DECLARED:
        p, i32, dp = ctypes.c_void_p, ctypes.c_int32, ctypes.POINTER(ctypes.c_double)
        ip = ctypes.POINTER(ctypes.c_int32)
        L.actune_tree_create.argtypes = [ip, dp, ip, ip, ip, i32, i32, i32, ctypes.POINTER(p)]
        L.actune_tree_create.restype = ctypes.c_int
        L.actune_tree_destroy.argtypes = [p]
        L.actune_tree_destroy.restype = None
        L.actune_tree_route_batch.argtypes = [p, dp, ctypes.POINTER(ctypes.c_uint8), dp, i32, i32, ip, ip]
        L.actune_tree_route_batch.restype = ctypes.c_int
        L.actune_action_features.argtypes = [dp, i32, ctypes.c_double, dp]
        L.actune_action_features.restype = ctypes.c_int
        _DECLARED = True
    return L


def _ptr(a, ctype):
    return None if a is None else a.ctypes.data_as(ctypes.POINTER(ctype))


@dataclass(frozen=True)
class Decision:
    region: str | None
    configuration: str


def action_forecast_features(actions, *, gripper_margin: float) -> dict:
    """The 13 causal features of one [H, 7] action chunk (features.py:46-96)."""
    chunk = np.asarray(actions, dtype=np.float64)
    if chunk.ndim != 2 or chunk.shape[1] != 7 or len(chunk) < 1:
        raise ValueError(f"expected a nonempty [H,7] action chunk, got {chunk.shape}")
    chunk = np.ascontiguousarray(chunk)
    out = np.empty(13, np.float64)
    rc = _lib_router().actune_action_features(_ptr(chunk, ctypes.c_double), len(chunk), float(gripper_margin),
                                              _ptr(out, ctypes.c_double))
    if rc != 0:
        raise ValueError("action chunk and gripper margin must be finite")
    return dict(zip(ACTION_FORECAST_FEATURE_NAMES, out.tolist()))


class PrecisionTree:
    def __init__(self, tree, state_dim, *, fallback="q11"):
        if not isinstance(state_dim, int) or not 1 <= state_dim <= MAX_STATE_DIM or fallback not in CONFIGURATIONS:
            raise ValueError("Invalid tree dimensions or fallback")
        self.tree = json.loads(json.dumps(tree))  # a private copy, like the reference's deepcopy
        self.state_dim, self.fallback = state_dim, fallback
        feature, threshold, left, right, profile, regions = [], [], [], [], [], []

        def flatten(t, region, depth):
            if depth > 5 or not isinstance(t, dict) or t.get("profile_index") not in range(4):
                raise ValueError("Invalid tree depth or configuration index")
            i = len(feature)
            feature.append(-1)
            threshold.append(0.0)
            left.append(-1)
            right.append(-1)
            profile.append(int(t["profile_index"]))
            regions.append(region)
            if "left" in t:
                f, thr = t.get("feature"), t.get("threshold", np.nan)
                if (not isinstance(f, int) or not 0 <= f < 13 + state_dim or "right" not in t
                        or not np.isfinite(thr)):
                    raise ValueError("Invalid tree split")
                feature[i], threshold[i] = f, float(thr)
                left[i] = flatten(t["left"], region + "/left", depth + 1)
                right[i] = flatten(t["right"], region + "/right", depth + 1)
            elif "right" in t:
                raise ValueError("Incomplete tree split")
            return i

        flatten(self.tree, "root", 0)
        self._regions = regions
        arrays = [np.asarray(feature, np.int32), np.asarray(threshold, np.float64), np.asarray(left, np.int32),
                  np.asarray(right, np.int32), np.asarray(profile, np.int32)]
        handle = ctypes.c_void_p()
        rc = _lib_router().actune_tree_create(
            _ptr(arrays[0], ctypes.c_int32), _ptr(arrays[1], ctypes.c_double), _ptr(arrays[2], ctypes.c_int32),
            _ptr(arrays[3], ctypes.c_int32), _ptr(arrays[4], ctypes.c_int32), len(feature), state_dim,
            CONFIGURATIONS.index(fallback), ctypes.byref(handle))
        if rc != 0:
            raise ValueError("Invalid tree")
        self._handle = handle

    def __del__(self):
        handle = getattr(self, "_handle", None)
        if handle is not None and handle.value:
            _lib_router().actune_tree_destroy(handle)
            self._handle = None

    def route_batch(self, features, states, has_history=None):
        """Configuration indices (into CONFIGURATIONS) and leaf nodes (-1: fallback)
        for a batch: features [B, 13] or None, states [B, S]."""
        states = np.ascontiguousarray(np.asarray(states, np.float64))
        if states.ndim != 2:
            raise ValueError("states must be [batch, state_dim]")
        batch = states.shape[0]
        feats = None if features is None else np.ascontiguousarray(np.asarray(features, np.float64))
        if feats is not None and feats.shape != (batch, 13):
            raise ValueError("features must be [batch, 13]")
        hist = None if has_history is None else np.ascontiguousarray(np.asarray(has_history, np.uint8))
        conf = np.empty(batch, np.int32)
        leaf = np.empty(batch, np.int32)
        rc = _lib_router().actune_tree_route_batch(self._handle, _ptr(feats, ctypes.c_double),
                                                   _ptr(hist, ctypes.c_uint8), _ptr(states, ctypes.c_double),
                                                   states.shape[1], batch, _ptr(conf, ctypes.c_int32),
                                                   _ptr(leaf, ctypes.c_int32))
        if rc != 0:
            raise ValueError("routing failed")
        return conf, leaf

    def _decision(self, conf, leaf):
        return Decision(None if leaf < 0 else self._regions[leaf], CONFIGURATIONS[conf])

    def route_vector(self, x):
        x = np.asarray(x, float)
        if x.shape != (13 + self.state_dim,):
            return Decision(None, self.fallback)
        conf, leaf = self.route_batch(x[None, :13], x[None, 13:])
        return self._decision(int(conf[0]), int(leaf[0]))

    def route(self, previous_features, state):
        if previous_features is None:
            return Decision(None, self.fallback)
        try:
            state = np.asarray(state, float).reshape(-1)
            if len(state) != self.state_dim:
                return Decision(None, self.fallback)
            x = np.r_[[previous_features[k] for k in ACTION_FORECAST_FEATURE_NAMES], state]
            return self.route_vector(x)
        except (KeyError, TypeError, ValueError):
            return Decision(None, self.fallback)

    def save(self, path):
        Path(path).write_text(json.dumps(dict(schema="actune_precision_tree_v1", tree=self.tree,
                                              state_dim=self.state_dim, fallback=self.fallback,
                                              configurations=CONFIGURATIONS), indent=2, allow_nan=False) + "\n")

    @classmethod
    def load(cls, path):
        data = json.loads(Path(path).read_text())
        if data.get("schema") != "actune_precision_tree_v1" or tuple(data["configurations"]) != CONFIGURATIONS:
            raise ValueError("Unsupported tree artifact")
        return cls(data["tree"], data["state_dim"], fallback=data["fallback"])


def random_selector_tree(rng, state_dim, *, leaves=3, max_depth=5, thresholds=None):
    """A random binary selector tree with `leaves` leaves (depth <= max_depth) over
    the 13 action features and `state_dim` state values.  Splits pick a random
    input and a threshold from `thresholds[input]` (a callable rng -> value) or a
    standard normal draw; leaves take distinct configurations while they last."""
    if not 1 <= leaves <= 2 ** max_depth:
        raise ValueError("leaves")
    configs = list(rng.permutation(4))
    root = {"profile_index": int(configs[0])}
    frontier = [(root, 0)]
    count = 1
    while count < leaves:
        splittable = [(n, d) for n, d in frontier if d < max_depth]
        node, depth = splittable[int(rng.integers(len(splittable)))]
        frontier.remove((node, depth))
        feature = int(rng.integers(13 + state_dim))
        thr = float(thresholds[feature](rng)) if thresholds and feature in thresholds else float(rng.standard_normal())
        left = {"profile_index": node["profile_index"]}
        right = {"profile_index": int(configs[count % 4])}
        node.update(feature=feature, threshold=thr, left=left, right=right)
        frontier += [(left, depth + 1), (right, depth + 1)]
        count += 1
    return root
