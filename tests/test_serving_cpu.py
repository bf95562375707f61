"""Serving host logic on the CPU: routing with a minimum dwell, grouping by
configuration, and a group of replica processes in which one replica leaves
between rounds (and, separately, one stops reporting) while the others carry on.
The policy here is a deterministic numpy stand-in; no GPU is involved."""
import multiprocessing as mp
import socket

import numpy as np
import pytest


def _tree_on_state0():
    from actune_b200.router import PrecisionTree
    # state[0] <= 0 -> q01 (index 1), else q10 (index 3)
    return PrecisionTree({"profile_index": 2, "feature": 13, "threshold": 0.0, "left": {"profile_index": 1},
                          "right": {"profile_index": 3}}, 14)


def fake_policy(config, envs, size, horizon=50):
    rng = np.random.default_rng(len(envs) * 31 + "q00q01q11q10".index(config))
    a = rng.normal(0, 0.1, (size, horizon, 32))
    return a[: len(envs)]


def test_dwell_delays_switches_by_two_requests():
    from actune_b200.serving import EnvRouter, serve_round
    router = EnvRouter(_tree_on_state0(), envs=4)
    seen = []
    for r in range(8):
        states = np.zeros((4, 14))
        states[:, 0] = -1.0 if (r // 3) % 2 == 0 else 1.0
        configs, actions = serve_round(fake_policy, router, states, buckets=(4,))
        assert actions.shape == (4, 50, 32)
        seen.append(int(configs[0]))
    # request 0: no history -> fallback q11 (2); the first switch waits for two
    # requests at the current configuration, later flips likewise.
    assert seen[0] == 2 and seen[1] == 2 and seen[2] == 1
    assert seen[3] == 1 and seen[4] == 3
    assert all(c in (1, 2, 3) for c in seen)
    assert router.switches >= 2


def test_groups_are_padded_to_buckets():
    from actune_b200.serving import groups_by_configuration
    groups = groups_by_configuration(np.array([0, 2, 2, 1, 2, 0, 2, 2, 2]), (4, 8, 16))
    assert [(c, list(e), s) for c, e, s in groups] == [(0, [0, 5], 4), (1, [3], 4), (2, [1, 2, 4, 6, 7, 8], 8)]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _replica(rank, world, port, rounds, mode, q):
    import os
    import time
    import torch.distributed as dist
    from actune_b200.serving import EnvRouter, ReplicaGroup, serve_round
    store = dist.TCPStore("127.0.0.1", port, world, is_master=rank == 0, timeout=__import__("datetime").timedelta(
        seconds=30))
    group = ReplicaGroup(store, rank, world)
    router = EnvRouter(_tree_on_state0(), envs=16)
    rng = np.random.default_rng(rank)
    t0 = time.perf_counter()
    chunks = 0
    for r in range(rounds):
        if rank == world - 1 and r == 2:
            if mode == "leave":
                group.leave(r, chunks, time.perf_counter() - t0)
                return
            os._exit(0)  # stops without a word: the others must not wait for it
        serve_round(fake_policy, router, rng.standard_normal((16, 14)), buckets=(4, 8, 16))
        chunks += 16
        group.heartbeat(r)
    group.finish(chunks, time.perf_counter() - t0)
    if rank == 0:
        q.put(group.collect(timeout_s=5.0))
        time.sleep(0.5)  # keep the store up while the others read it


@pytest.mark.parametrize("mode", ["leave", "vanish"])
def test_replica_leaving_between_rounds_does_not_stop_the_others(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port, world, rounds = _free_port(), 3, 6
    procs = [ctx.Process(target=_replica, args=(r, world, port, rounds, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    report = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert sorted(report["finished"]) == [0, 1]
    assert all(v["chunks"] == 16 * rounds for v in report["finished"].values())
    if mode == "leave":
        assert list(report["left"]) == [2] and report["left"][2]["chunks"] == 32 and report["silent"] == []
    else:
        assert report["left"] == {} and report["silent"] == [2]
    assert report["chunks_per_s"] > 0
