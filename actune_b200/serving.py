"""Serving independent environments with per-request precision routing.

A replica owns one GPU and serves a batch of environments.  Every request round:

1. each environment's configuration is routed by the selector tree
   (``router.PrecisionTree``) from the 13 features of its previous action chunk and
   its proprioceptive state -- the reference's ``Controller.predict``
   (actune/runtime.py:67-108) does this per request;
2. a configuration change takes effect only after the environment has spent at
   least two requests at its current one (the minimum dwell the benchmark
   configuration asks for on precision; the reference applies its dwell to the
   hardware operating point, runtime.py:100);
3. environments sharing a configuration run as one batched policy call under
   ``precision_profile`` (padded to a fixed batch bucket, so each bucket and
   configuration replays its own CUDA graph);
4. the actions come back to the host and their features feed the next routing.

Replicas are independent (no data-path collective).  ``ReplicaGroup`` keeps the
host-side bookkeeping of a group of replicas in a key-value store: heartbeats per
round, an explicit ``leave`` between rounds, and the aggregate of the replicas
that finished -- a replica that left or stopped reporting is named, not waited
for.
"""
from __future__ import annotations

import json
import time
from dataclasses import dataclass, field

import numpy as np

from .precision import CONFIGURATIONS
from .router import action_forecast_features

MIN_DWELL = 2


@dataclass
class EnvRouter:
    """Per-environment routing state: current configuration, requests spent at it,
    and the features of the previous chunk (None before the first)."""

    tree: object
    envs: int
    fallback: str = "q11"
    current: np.ndarray = field(init=False)
    dwell: np.ndarray = field(init=False)
    features: np.ndarray | None = field(init=False, default=None)

    def __post_init__(self):
        self.current = np.full(self.envs, CONFIGURATIONS.index(self.fallback), np.int32)
        self.dwell = np.zeros(self.envs, np.int32)
        self.switches = 0

    def assign(self, states):
        """Configuration index per environment for this request (routing + dwell)."""
        routed, _ = self.tree.route_batch(self.features, states)
        change = (routed != self.current) & (self.dwell >= MIN_DWELL)
        self.current = np.where(change, routed, self.current).astype(np.int32)
        self.dwell = np.where(change, 0, self.dwell)
        self.switches += int(change.sum())
        return self.current.copy()

    def observe(self, actions, gripper_dim=6):
        """Features of each environment's new chunk ([envs, H, >=7] actions; the
        first 7 dimensions are the arm and gripper command, the gripper margin is
        the smallest distance of the gripper command from its switching point)."""
        feats = np.empty((self.envs, 13))
        for e in range(self.envs):
            a = np.asarray(actions[e, :, :7], np.float64)
            f = action_forecast_features(a, gripper_margin=float(np.abs(a[:, gripper_dim]).min()))
            feats[e] = list(f.values())
        self.features = feats
        self.dwell += 1


def groups_by_configuration(configs, buckets):
    """[(configuration index, env indices, padded batch size)] for one request."""
    out = []
    for c in np.unique(configs):
        envs = np.flatnonzero(configs == c)
        size = next(b for b in buckets if b >= len(envs))
        out.append((int(c), envs, size))
    return out


def serve_round(policy, router, states, buckets):
    """One request round for every environment.  `policy(config_name, env_indices,
    padded_size)` returns host actions [len(env_indices), H, D]."""
    configs = router.assign(states)
    actions = None
    for c, envs, size in groups_by_configuration(configs, buckets):
        out = policy(CONFIGURATIONS[c], envs, size)
        if actions is None:
            actions = np.empty((router.envs,) + out.shape[1:], out.dtype)
        actions[envs] = out
    router.observe(actions)
    return configs, actions


class ReplicaGroup:
    """Host-side bookkeeping of independent replicas in a key-value store
    (``torch.distributed.Store``: set / get / check / add)."""

    def __init__(self, store, rank, world, prefix="serving"):
        self.store, self.rank, self.world, self.prefix = store, rank, world, prefix

    def _k(self, *parts):
        return "/".join([self.prefix, *map(str, parts)])

    def heartbeat(self, round_index):
        self.store.set(self._k("beat", self.rank), str(round_index))

    def leave(self, round_index, chunks, seconds):
        """Leave the group between rounds, reporting what was served."""
        self.store.set(self._k("left", self.rank), json.dumps({"round": round_index, "chunks": chunks,
                                                               "seconds": seconds}))

    def finish(self, chunks, seconds, **extra):
        self.store.set(self._k("done", self.rank), json.dumps({"chunks": chunks, "seconds": seconds, **extra}))

    def collect(self, timeout_s=30.0, poll_s=0.05):
        """Wait (up to timeout_s) for every replica to finish or leave.  Returns
        {"finished": {rank: report}, "left": {rank: report}, "silent": [ranks],
        "chunks_per_s": aggregate of the finished replicas}."""
        deadline = time.monotonic() + timeout_s
        finished, left = {}, {}
        while True:
            for r in range(self.world):
                if r in finished or r in left:
                    continue
                if self.store.check([self._k("done", r)]):
                    finished[r] = json.loads(self.store.get(self._k("done", r)))
                elif self.store.check([self._k("left", r)]):
                    left[r] = json.loads(self.store.get(self._k("left", r)))
            if len(finished) + len(left) == self.world or time.monotonic() > deadline:
                break
            time.sleep(poll_s)
        silent = [r for r in range(self.world) if r not in finished and r not in left]
        rate = sum(v["chunks"] / v["seconds"] for v in finished.values() if v["seconds"] > 0)
        return {"finished": finished, "left": left, "silent": silent, "chunks_per_s": rate}
