"""Row-sharded training on 2+ GPUs (one process per GPU, NCCL communicator)
through libdp_gbdt: every rank must hold the same model, equal to the CPU
oracle's on all rows, and every rank's margins must equal the oracle's margins
of its rows.  Skipped on a box with fewer than two GPUs."""
import json
import os
import socket
import subprocess
import sys
import pathlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
ROOT = pathlib.Path(__file__).resolve().parents[1]


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs at least two GPUs")
@pytest.mark.parametrize("case,K", [("squared", 1), ("logistic_nan", 1), ("softprob", 4), ("deep_exact_host", 1),
                                    ("sampled", 1), ("wide", 1)])
def test_sharded_ranks_match_the_oracle(orc, tmp_path, case, K):
    import _multi_gpu_worker as w
    world = min(torch.cuda.device_count(), 4)
    rounds = 4
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    if case == "deep_exact_host":
        # host matrices; levels past 3 open nodes read exact counts back first
        env.update(DP_ASYNC_OPEN_LIMIT="3", DP_ASYNC_HIST_BYTES=str(8 * 24 * 256 * 16))
    if case == "wide":
        env.update(DP_HIST_WIDE="1")  # the 64-feature histogram kernel with sharded rows
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={free_port()}",
           str(ROOT / "tests" / "_multi_gpu_worker.py"), case, str(tmp_path), str(rounds)]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    models = [(tmp_path / f"rank{k}.json").read_bytes() for k in range(world)]
    assert all(m == models[0] for m in models)
    x, y, params = w.data(case)
    sampling = {k: params[k] for k in ("subsample", "colsample_bytree", "colsample_bylevel", "colsample_bynode",
                                        "seed") if k in params}
    o = orc.Model(x, y, params["objective"], num_class=K, max_depth=params["max_depth"], rounds=rounds, threads=8,
                  min_child_weight=params.get("min_child_weight", 1.0), **sampling)
    trees = json.loads(models[0])["learner"]["gradient_booster"]["model"]["trees"]
    assert len(trees) == o.num_trees()
    for i, t in enumerate(trees):
        ot = o.tree(i)
        for f in ("left_children", "right_children", "split_indices"):
            np.testing.assert_array_equal(np.array(t[f]), ot[f])
        for f in ("split_conditions", "base_weights", "sum_hessian"):
            np.testing.assert_array_equal(np.array(t[f], np.float32).view(np.uint32), ot[f].view(np.uint32))
    margins = np.concatenate([np.load(tmp_path / f"rank{k}_margins.npy") for k in range(world)])
    np.testing.assert_array_equal(margins.view(np.uint32), o.margins().view(np.uint32))

