"""Golden vectors for the per-request router, made by running the reference's
own code (actune/tree.py PrecisionTree.route_vector / route and
actune/features.py action_forecast_features) on seeded random trees, inputs and
action chunks.  Run in the build container, where the reference is mounted:

    python tests/golden/gen_router.py [/path/to/reference]

Writes tests/golden/router.npz (inputs, configurations, regions, features)."""
import json
import sys
from pathlib import Path

import numpy as np

REF = Path(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
sys.path.insert(0, str(REF))
from actune.features import action_forecast_features  # noqa: E402
from actune.tree import CONFIGURATIONS, PrecisionTree  # noqa: E402

STATE = 14
rng = np.random.default_rng(0)


def random_tree(leaves):
    root = {"profile_index": int(rng.integers(4))}
    frontier = [(root, 0)]
    for _ in range(leaves - 1):
        node, depth = frontier.pop(int(rng.integers(len([f for f in frontier if f[1] < 5]))))
        f = int(rng.integers(13 + STATE))
        thr = float(rng.uniform(0, 1)) if f < 13 else float(rng.standard_normal())
        node.update(feature=f, threshold=thr, left={"profile_index": int(rng.integers(4))},
                    right={"profile_index": int(rng.integers(4))})
        frontier += [(node["left"], depth + 1), (node["right"], depth + 1)]
        frontier = [x for x in frontier if x[1] <= 5]
    return root


trees, xs, confs, regions, tree_of = [], [], [], [], []
for t in range(24):
    tree = random_tree(int(rng.integers(1, 9)))
    pt = PrecisionTree(tree, STATE, fallback=CONFIGURATIONS[t % 4])
    trees.append({"tree": tree, "fallback": CONFIGURATIONS[t % 4]})
    for i in range(60):
        x = np.r_[rng.uniform(0, 1, 13), rng.standard_normal(STATE)]
        if i % 15 == 7:
            x[int(rng.integers(len(x)))] = np.nan
        if i % 20 == 11:
            x[int(rng.integers(len(x)))] = np.inf
        d = pt.route_vector(x)
        xs.append(x)
        confs.append(CONFIGURATIONS.index(d.configuration))
        regions.append(d.region if d.region is not None else "")
        tree_of.append(t)

chunks, margins, feats, horizons = [], [], [], []
for i in range(48):
    H = [1, 2, 3, 7, 8, 9, 16, 50][i % 8]
    a = rng.normal(0, 0.1, (H, 7))
    a[:, 6] = rng.choice([-1.0, 0.0, 1.0], H) * (i % 3 != 0) + (i % 3 == 0) * np.sign(rng.standard_normal()) * 0.5
    if i % 12 == 5:
        a[:, :6] = 0.0
    m = float(rng.uniform(0, 1))
    f = action_forecast_features(a, gripper_margin=m)
    pad = np.zeros((50, 7))
    pad[:H] = a
    chunks.append(pad)
    horizons.append(H)
    margins.append(m)
    feats.append([f[k] for k in f])

out = Path(__file__).with_name("router.npz")
np.savez_compressed(out, x=np.asarray(xs), configuration=np.asarray(confs, np.int32),
                    tree_of=np.asarray(tree_of, np.int32), regions=np.asarray(regions),
                    trees=np.asarray(json.dumps(trees)), chunks=np.asarray(chunks),
                    horizons=np.asarray(horizons, np.int32), margins=np.asarray(margins),
                    features=np.asarray(feats), feature_names=np.asarray(list(f.keys())))
print(out, len(xs), "routes,", len(feats), "chunks")
