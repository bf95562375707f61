"""Serving on the GPU (config 4's host loop over the pi0.5 policy, small shapes).

* A batched chunk (several environments padded to a bucket, one CUDA graph per
  bucket, step shape and configuration) gives every environment exactly the
  actions it gets when served alone, eagerly.
* A few request rounds through the router, the dwell and the grouping serve every
  environment once per round, and the bank audit sees each request.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPE = dict(vlm_layers=2, vlm_hidden=256, vlm_mlp=512, expert_layers=2, expert_hidden=256, expert_mlp=256,
             heads=4, kv_heads=1, head_dim=64, horizon=8, action_dim=8)


@pytest.fixture(scope="module")
def serving():
    from actune_b200.harness import Pi05Serving
    s = Pi05Serving(envs=6, buckets=(2, 4, 8), seed=3, **SHAPE)
    yield s
    s.release()


def test_batched_chunk_matches_single_environment_eager(serving):
    from actune_b200.harness import sample_pi05
    from actune_b200.precision import precision_profile
    g = torch.Generator().manual_seed(1)
    images = torch.randint(0, 256, (6, 224, 224, 3), generator=g, dtype=torch.uint8).cuda()
    states = torch.randn(6, 14, generator=g).cuda()
    rows = np.array([1, 3, 4])
    for config in ("q00", "q11"):
        batched = serving.chunk(config, images, states, rows, 4)
        for j, e in enumerate(rows):
            with precision_profile(config), torch.inference_mode():
                single = sample_pi05(serving.model, serving._prefix, serving.model.denoise_step,
                                     images[e:e + 1], serving.noise[j:j + 1], states[e:e + 1])
            assert torch.equal(batched[j:j + 1], single), (config, e)
    assert serving.prefix.replays >= 1 and serving.step.replays >= 10


def test_request_rounds_route_group_and_audit(serving):
    from actune_b200.router import PrecisionTree
    from actune_b200.serving import EnvRouter, serve_round
    tree = PrecisionTree({"profile_index": 2, "feature": 13, "threshold": 0.0, "left": {"profile_index": 0},
                          "right": {"profile_index": 3}}, 14)
    router = EnvRouter(tree, 6)
    g = torch.Generator().manual_seed(2)
    images = torch.randint(0, 256, (6, 224, 224, 3), generator=g, dtype=torch.uint8).cuda()
    serving.runtime.before()

    def policy(config, envs, size):
        states_dev = torch.from_numpy(states).float().cuda()
        return serving.chunk(config, images, states_dev, envs, size).cpu().numpy()

    used = set()
    for r in range(5):
        states = np.random.default_rng(r).standard_normal((6, 14))
        configs, actions = serve_round(policy, router, states, serving.buckets)
        used |= set(configs.tolist())
        assert actions.shape == (6, 8, 8) and np.isfinite(actions).all()
    assert 2 in used and len(used) >= 2           # fallback first, routed configurations after the dwell
    calls = {n: m.calls for n, m in serving.runtime.modules.items()}
    assert all(c > 0 for c in calls.values())
    from actune_b200 import _lib
    assert _lib.device_error() == (0, 0)
