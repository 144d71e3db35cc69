"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (configs 1-4), full size for config 1 and scaled
down for configs 2-4 so that the CPU oracle trains them in seconds.  Shared
by make_config_fixtures.py and the tests that check its fixtures."""
from __future__ import annotations

import numpy as np

CONFIGS = {
    # name: (generator, objective, num_class, max_depth, rounds)
    "config1": ("c1", "binary:logistic", 1, 4, 20),
    "config2_small": ("c2", "binary:logistic", 1, 8, 5),
    "config3_small": ("c3", "multi:softprob", 10, 6, 2),
    "config4_small": ("c4", "reg:squarederror", 1, 10, 3),
}
SEED = 4242


def c1(seed: int = SEED):
    """Config 1 at full size: 20,000 x 16 N(0,1); y = 1[x0 + 0.5 x1 x2 + N(0, 0.3) > 0]."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((20_000, 16)).astype(np.float32)
    y = (x[:, 0] + 0.5 * x[:, 1] * x[:, 2] + rng.normal(0.0, 0.3, 20_000) > 0).astype(np.float32)
    return x, y


def c2(seed: int = SEED + 2, rows: int = 20_000):
    """Config 2 scaled to 20,000 rows: 64 columns (32 N(0,1), 32 U(0,1));
    label = sign of a seeded sparse linear-plus-pairwise teacher about its
    median, 10% of labels flipped."""
    rng = np.random.default_rng(seed)
    x = np.concatenate([rng.standard_normal((rows, 32)), rng.random((rows, 32))], 1).astype(np.float32)
    lin = rng.choice(64, 12, replace=False)
    w = rng.normal(0.0, 1.0, 12)
    pairs = rng.choice(64, (6, 2))
    c = rng.normal(0.0, 1.0, 6)
    score = x[:, lin].astype(np.float64) @ w
    for (i, j), cf in zip(pairs, c):
        score += cf * x[:, i].astype(np.float64) * x[:, j]
    y = (score > np.median(score)).astype(np.float32)
    flip = rng.random(rows) < 0.1
    y[flip] = 1.0 - y[flip]
    return x, y


def c3(seed: int = SEED + 3, rows: int = 3_000):
    """Config 3 scaled to 3,000 rows: 784 uint8 values, 80% zeros, non-zeros
    Uniform{1..255}; 10 classes = argmax of a seeded linear teacher."""
    rng = np.random.default_rng(seed)
    nz = rng.random((rows, 784)) < 0.2
    v = rng.integers(1, 256, (rows, 784))
    x = np.where(nz, v, 0).astype(np.float32)
    w = rng.standard_normal((784, 10))
    y = np.argmax(x.astype(np.float64) @ w, 1).astype(np.float32)
    return x, y


def c4(seed: int = SEED + 4, rows: int = 20_000):
    """Config 4 scaled to 20,000 rows: 128 N(0,1) features; target = a seeded
    random depth-6, 20-tree ensemble plus N(0, 0.1)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, 128)).astype(np.float32)
    feats = rng.integers(0, 128, (20, 63))
    thr = rng.normal(0.0, 0.7, (20, 63)).astype(np.float32)
    leaf = rng.normal(0.0, 1.0, (20, 64))
    y = np.zeros(rows)
    for t in range(20):
        idx = np.zeros(rows, np.int64)
        for _ in range(6):
            f = feats[t][idx]
            go = (x[np.arange(rows), f] >= thr[t][idx]).astype(np.int64)
            idx = 2 * idx + 1 + go
        y += leaf[t][idx - 63]
    y += rng.normal(0.0, 0.1, rows)
    return x, y.astype(np.float32)


def data(name: str):
    gen = CONFIGS[name][0]
    return {"c1": c1, "c2": c2, "c3": c3, "c4": c4}[gen]()


def tree_digest(trees) -> str:
    """sha256 over every tree's left, right, split index (int32), default_left
    (uint8) and split condition (float32, leaf values at leaves), in order.
    `trees` holds dicts with the model JSON's field names."""
    import hashlib
    h = hashlib.sha256()
    for t in trees:
        for f in ("left_children", "right_children", "split_indices"):
            h.update(np.asarray(t[f], dtype="<i4").tobytes())
        h.update(np.asarray(t["default_left"], dtype=np.uint8).tobytes())
        h.update(np.asarray(t["split_conditions"], dtype="<f4").tobytes())
    return h.hexdigest()


def array_digest(a) -> str:
    import hashlib
    return hashlib.sha256(np.ascontiguousarray(a, dtype="<f4").tobytes()).hexdigest()
