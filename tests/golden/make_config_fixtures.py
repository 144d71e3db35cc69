"""Frozen outputs of the CPU oracle on the benchmark configurations (config 1
at full size, configs 2-4 scaled down), with the seeds and generators of
config_data.py:

    python tests/golden/make_config_fixtures.py

The fixture (configs/frozen.json) holds, per configuration, digests of the cuts,
of every tree (structure, split features, default directions, fp32
thresholds and leaf values) and of the training margins, plus the node
counts and the root split of each tree.  The CPU oracle must keep producing
them (tests/test_oracle.py) and the CUDA path must produce the same trees and
margins (tests/test_gpu_train.py).  They pin the oracle to its own earlier
outputs; its independent pins are the fixtures of make_golden.py."""
from __future__ import annotations

import hashlib
import json
import pathlib
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(HERE.parents[1] / "oracle"))

import config_data  # noqa: E402
import oracle  # noqa: E402


def oracle_fixture(name: str) -> dict:
    _, objective, K, depth, rounds = config_data.CONFIGS[name]
    x, y = config_data.data(name)
    m = oracle.Model(x, y, objective, num_class=K, max_depth=depth, max_bin=256, eta=0.3, rounds=rounds,
                     threads=oracle.default_threads())
    trees = [m.tree(i) for i in range(m.num_trees())]
    cut, nb, hm = m.cuts()
    hc = hashlib.sha256()
    for f in range(x.shape[1]):
        hc.update(np.asarray(cut[f][: max(int(nb[f]) - 1, 0)], dtype="<f4").tobytes())
    hc.update(np.asarray(nb, dtype="<u2").tobytes())
    hc.update(np.asarray(hm, dtype=np.uint8).tobytes())
    return {
        "rows": int(x.shape[0]), "features": int(x.shape[1]), "objective": objective, "num_class": K,
        "max_depth": depth, "rounds": rounds, "max_bin": 256, "eta": 0.3,
        "cuts_sha256": hc.hexdigest(),
        "trees_sha256": config_data.tree_digest(trees),
        "margins_sha256": config_data.array_digest(m.margins()),
        "nodes_per_tree": [int(len(t["left_children"])) for t in trees],
        "root_splits": [[int(t["split_indices"][0]), float(t["split_conditions"][0])] for t in trees],
    }


def main() -> None:
    out = {name: oracle_fixture(name) for name in config_data.CONFIGS}
    (HERE / "configs" / "frozen.json").write_text(json.dumps(out, indent=1) + "\n")


if __name__ == "__main__":
    main()
