"""Row-sharded training on CPU ranks (gloo): the algorithm the multi-GPU path
runs -- radix-selection cuts from summed counts, quantiser maxima over ranks,
summed integer histograms, child sizes from summed counts -- must grow the
same trees as one rank on all rows.  Also checks, on one process, that the
radix-selection cut search equals the sort-based cut rule."""
import socket

import numpy as np
import pytest


def special_matrix(R, F, seed, nan_frac=0.0):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((R, F)).astype(np.float32)
    x[:, 1] = rng.integers(0, 5, R)
    x[:, 2] = 3.0
    x[:, 3] = np.where(rng.random(R) < 0.5, -0.0, 0.0)
    x[: R // 3, 3] = rng.standard_normal(R // 3)
    x[:, 4] = rng.integers(0, 256, R)
    x[:, 5] = np.nan
    x[:, 6] = rng.integers(0, 255, R)
    x[rng.random(R) < 0.1, 6] = np.nan
    x[:, 7] = np.round(rng.standard_normal(R) * 4) / 4
    if nan_frac:
        x[rng.random((R, F)) < nan_frac] = np.nan
    return x


@pytest.mark.parametrize("R,F,max_bin,nan_frac", [(1, 9, 256, 0.0), (7, 9, 256, 0.0), (5000, 12, 256, 0.05),
                                                  (30000, 16, 256, 0.0), (20000, 9, 16, 0.0), (3000, 40, 64, 0.2)])
def test_radix_selection_equals_sort_rule(orc, R, F, max_bin, nan_frac):
    x = special_matrix(R, F, R + F, nan_frac) if F >= 8 else np.random.default_rng(0).standard_normal((R, F))
    cut, nb, hm = orc.cuts(x, max_bin)
    rcut, rnb, rhm = orc.radix_cuts(x, max_bin)
    np.testing.assert_array_equal(rnb, nb)
    np.testing.assert_array_equal(rhm, hm)
    np.testing.assert_array_equal(rcut.view(np.uint32), cut.view(np.uint32))


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("objective,K,nan_frac", [("reg:squarederror", 1, 0.0), ("binary:logistic", 1, 0.1),
                                                  ("multi:softprob", 3, 0.0)])
def test_two_gloo_ranks_grow_the_trees_of_one_rank(orc, objective, K, nan_frac):
    import _gloo_worker
    import torch.multiprocessing as mp

    rng = np.random.default_rng(7)
    R, F = 6001, 10
    x = rng.standard_normal((R, F)).astype(np.float32)
    if nan_frac:
        x[rng.random((R, F)) < nan_frac] = np.nan
    signal = np.nan_to_num(x[:, 0]) + 0.5 * np.nan_to_num(x[:, 1])
    if objective == "binary:logistic":
        y = (signal > 0).astype(np.float32)
    elif K > 1:
        y = np.digitize(signal, [-0.5, 0.5]).astype(np.float32)
    else:
        y = (signal + 0.1 * rng.standard_normal(R)).astype(np.float32)
    kw = dict(objective=objective, num_class=K, max_depth=5, rounds=3, threads=2)
    # the manager's server process is spawned too: forking a process that
    # already runs threads (the oracle's, OpenMP's) can deadlock the child
    with mp.get_context("spawn").Manager() as manager:
        out = manager.dict()
        mp.spawn(_gloo_worker.run, args=(2, free_port(), x, y, kw, out), nprocs=2, join=True)
        got = dict(out)
    ref = orc.Model(x, y, **kw)
    ref_cut, ref_nb, ref_hm = ref.cuts()
    for rank in (0, 1):
        cut, nb, hm = got[rank]["cuts"]
        np.testing.assert_array_equal(nb, ref_nb)
        np.testing.assert_array_equal(cut.view(np.uint32), ref_cut.view(np.uint32))
        assert len(got[rank]["trees"]) == ref.num_trees()
        for i, t in enumerate(got[rank]["trees"]):
            for key, v in ref.tree(i).items():
                np.testing.assert_array_equal(t[key], v, err_msg=f"rank {rank} tree {i} {key}")
    lo = R // 2
    np.testing.assert_array_equal(got[0]["margins"], ref.margins()[:lo])
    np.testing.assert_array_equal(got[1]["margins"], ref.margins()[lo:])
