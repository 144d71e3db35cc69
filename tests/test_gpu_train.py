"""End-to-end parity: trees grown through the XGBoost C-API subset
(XGBoosterUpdateOneIter, the call at native/class_native_training.cuh:67)
against the CPU oracle on the same seeded inputs.  Trees must be identical
field by field (structure, split features, fp32 thresholds, default
directions, leaf values, gains, hessian sums) and so must the training
margins."""
import json

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

FIELDS_EXACT = ["left_children", "right_children", "split_indices", "default_left"]
FIELDS_F32 = ["split_conditions", "base_weights", "loss_changes", "sum_hessian"]


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def compare_models(b, o, K):
    trees = b.trees()
    assert len(trees) == o.num_trees()
    for i, t in enumerate(trees):
        ot = o.tree(i)
        for f in FIELDS_EXACT:
            np.testing.assert_array_equal(np.array(t[f], np.int64), ot[f].astype(np.int64), err_msg=f"tree {i} {f}")
        for f in FIELDS_F32:
            got = np.array(t[f], np.float32)
            np.testing.assert_array_equal(got.view(np.uint32), ot[f].view(np.uint32), err_msg=f"tree {i} {f}")
    return trees


def run(dp, orc, x, y, objective, rounds, K=1, **hp):
    params = {"objective": objective, "tree_method": "hist", "device": "cuda:0", "max_depth": hp.get("max_depth", 6),
              "max_bin": hp.get("max_bin", 256), "eta": hp.get("eta", 0.3), "lambda": hp.get("reg_lambda", 1.0),
              "alpha": hp.get("alpha", 0.0), "gamma": hp.get("gamma", 0.0),
              "min_child_weight": hp.get("min_child_weight", 1.0)}
    if objective.startswith("multi:"):
        params["num_class"] = K
    d = dp.DMatrix.from_torch(cuda(x), cuda(y))
    b = dp.train(params, d, rounds)
    assert b.boosted_rounds() == rounds
    o = orc.Model(x, y, objective, num_class=K, max_depth=params["max_depth"], max_bin=params["max_bin"],
                  eta=params["eta"], reg_lambda=params["lambda"], alpha=params["alpha"], gamma=params["gamma"],
                  min_child_weight=params["min_child_weight"], rounds=rounds, threads=orc.default_threads())
    trees = compare_models(b, o, K)
    R = x.shape[0]
    np.testing.assert_array_equal(b.margins(R, K).view(np.uint32), o.margins().view(np.uint32))
    return b, o, trees


def c1_data(R=20000, seed=0):
    """x ~ N(0,1) 16 features; y = 1[x0 + 0.5 x1 x2 + N(0, 0.3) > 0]."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((R, 16), dtype=np.float32)
    y = (x[:, 0] + 0.5 * x[:, 1] * x[:, 2] + rng.normal(0, 0.3, R) > 0).astype(np.float32)
    return x, y


def test_config1_binary_logistic_full_size(dp, orc):
    x, y = c1_data()
    b, o, trees = run(dp, orc, x, y, "binary:logistic", 20, max_depth=4)
    assert len(trees) == 20 and all(len(t["left_children"]) <= 31 for t in trees)
    m = b.margins(len(y), 1)[:, 0]
    assert ((m > 0) == (y > 0.5)).mean() > 0.85


def test_squared_error_with_missing_values(dp, orc):
    rng = np.random.default_rng(3)
    R, F = 6000, 10
    x = rng.standard_normal((R, F)).astype(np.float32)
    y = (np.sin(x[:, 0]) + x[:, 1] ** 2 + 0.1 * rng.standard_normal(R)).astype(np.float32)
    x[rng.random((R, F)) < 0.2] = np.nan
    run(dp, orc, x, y, "reg:squarederror", 6, max_depth=5)


@pytest.mark.parametrize("objective", ["multi:softprob", "multi:softmax"])
def test_multiclass(dp, orc, objective):
    rng = np.random.default_rng(4)
    R, F, K = 4000, 30, 5
    x = rng.standard_normal((R, F)).astype(np.float32)
    w = rng.standard_normal((F, K))
    y = np.argmax(x @ w, 1).astype(np.float32)
    b, o, trees = run(dp, orc, x, y, objective, 3, K=K, max_depth=4)
    assert [t["id"] for t in trees] == list(range(15))
    doc = json.loads(b.save_raw())
    assert doc["learner"]["gradient_booster"]["model"]["tree_info"] == [0, 1, 2, 3, 4] * 3
    assert doc["learner"]["gradient_booster"]["model"]["iteration_indptr"] == [0, 5, 10, 15]


def test_config3_shape_uint8_sparse_multiclass(dp, orc):
    """BASELINE config 3 shape, scaled down: 784 uint8 features, 80% zeros, 10 classes."""
    rng = np.random.default_rng(5)
    R, F, K = 3000, 784, 10
    x = np.where(rng.random((R, F)) < 0.8, 0, rng.integers(1, 256, (R, F))).astype(np.float32)
    y = np.argmax(x @ rng.standard_normal((F, K)), 1).astype(np.float32)
    run(dp, orc, x, y, "multi:softprob", 2, K=K, max_depth=3)


@pytest.mark.parametrize("hp", [dict(alpha=0.5, gamma=1.0, min_child_weight=5.0, reg_lambda=2.0),
                                dict(max_bin=16, max_depth=7), dict(eta=1.0, reg_lambda=0.0, min_child_weight=0.0),
                                dict(max_depth=10)])
def test_regularisation_and_shapes(dp, orc, hp):
    x, y = c1_data(8000, seed=9)
    run(dp, orc, x, y, "binary:logistic", 4, **hp)


@pytest.mark.parametrize("objective,K", [("binary:logistic", 1), ("multi:softprob", 4)])
def test_deep_trees_with_exact_level_counts(dp, orc, monkeypatch, objective, K):
    """Levels whose open-node bound passes the limits read the exact counts
    back before sizing their buffers; trees stop growing at different depths."""
    monkeypatch.setenv("DP_ASYNC_OPEN_LIMIT", "3")
    monkeypatch.setenv("DP_ASYNC_HIST_BYTES", str(6 * 16 * 256 * 16))
    x, y = c1_data(3000, seed=11)
    if K > 1:
        y = np.digitize(x[:, 0] + x[:, 3], [-1.0, 0.0, 1.0]).astype(np.float32)
    run(dp, orc, x, y, objective, 3, K=K, max_depth=13, min_child_weight=0.0)


@pytest.mark.parametrize("wide", ["0", "1"])
def test_both_histogram_kernels_train_the_same_trees(dp, orc, monkeypatch, wide):
    """Training with the 32- or the 64-feature histogram kernel (DP_HIST_WIDE),
    a feature count that leaves the last tile partial, and missing values."""
    monkeypatch.setenv("DP_HIST_WIDE", wide)
    rng = np.random.default_rng(31)
    x = rng.standard_normal((9000, 100)).astype(np.float32)
    x[rng.random(x.shape) < 0.03] = np.nan
    y = (np.nan_to_num(x[:, 0]) + 0.5 * np.nan_to_num(x[:, 77]) + 0.2 * rng.standard_normal(9000)).astype(np.float32)
    run(dp, orc, x, y, "reg:squarederror", 3, max_depth=6)


def test_deep_trees_device_resident_levels(dp, orc):
    x, y = c1_data(6000, seed=12)
    run(dp, orc, x, y, "binary:logistic", 2, max_depth=14, min_child_weight=0.0, reg_lambda=0.1)


@pytest.mark.parametrize("graphs", ["0", "1"])
def test_direct_and_graph_rounds_agree(dp, orc, monkeypatch, graphs):
    """Rounds after the first replay a captured CUDA graph; with capture off
    (DP_CUDA_GRAPHS=0) every round is launched directly.  Both grow the
    oracle's trees, with the profiler on for part of the rounds."""
    monkeypatch.setenv("DP_CUDA_GRAPHS", graphs)
    x, y = c1_data(12000, seed=13)
    params = {"objective": "binary:logistic", "tree_method": "hist", "device": "cuda:0", "max_depth": 6,
              "max_bin": 256, "eta": 0.3}
    d = dp.DMatrix.from_torch(cuda(x), cuda(y))
    b = dp.Booster(params, [d])
    for i in range(6):
        if i == 3:
            b.set_profiling(True)
        b.update(d, i)
    prof = b.profile()
    assert prof["histograms"]["launches"] == 3 * 6 and prof["histograms"]["ms"] > 0
    o = orc.Model(x, y, "binary:logistic", max_depth=6, max_bin=256, eta=0.3, rounds=6, threads=8)
    compare_models(b, o, 1)
    np.testing.assert_array_equal(b.margins(len(y), 1).view(np.uint32), o.margins().view(np.uint32))


SAMPLING_CASES = [
    dict(subsample=0.6),
    dict(colsample_bytree=0.5),
    dict(colsample_bylevel=0.7),
    dict(colsample_bynode=0.4),
    dict(subsample=0.8, colsample_bytree=0.8, colsample_bylevel=0.75, colsample_bynode=0.6, seed=12345),
]


@pytest.mark.parametrize("sampling", SAMPLING_CASES)
@pytest.mark.parametrize("objective,K", [("binary:logistic", 1), ("multi:softprob", 3)])
def test_sampling_matches_oracle(dp, orc, sampling, objective, K):
    """Row and column sampling with the counter-based hash: the GPU path
    (rounds after the first replayed as a graph) grows the oracle's trees."""
    rng = np.random.default_rng(21)
    R, F = 7000, 23
    x = rng.standard_normal((R, F)).astype(np.float32)
    x[rng.random((R, F)) < 0.03] = np.nan
    s = np.nan_to_num(x[:, 0]) + 0.7 * np.nan_to_num(x[:, 3]) - 0.5 * np.nan_to_num(x[:, 11])
    y = (s > 0).astype(np.float32) if K == 1 else np.digitize(s, [-0.6, 0.6]).astype(np.float32)
    params = {"objective": objective, "tree_method": "hist", "device": "cuda:0", "max_depth": 5, "max_bin": 256,
              "eta": 0.3}
    if K > 1:
        params["num_class"] = K
    params.update({k: v for k, v in sampling.items()})
    d = dp.DMatrix.from_torch(cuda(x), cuda(y))
    b = dp.train(params, d, 4)
    o = orc.Model(x, y, objective, num_class=K, max_depth=5, max_bin=256, eta=0.3, rounds=4, threads=8,
                  **sampling)
    compare_models(b, o, K)
    np.testing.assert_array_equal(b.margins(R, K).view(np.uint32), o.margins().view(np.uint32))


@pytest.mark.parametrize("R", [1, 2, 7, 33])
def test_tiny_inputs(dp, orc, R):
    rng = np.random.default_rng(R)
    x = rng.standard_normal((R, 3)).astype(np.float32)
    y = rng.standard_normal(R).astype(np.float32)
    run(dp, orc, x, y, "reg:squarederror", 3, max_depth=4, min_child_weight=0.0)


@pytest.mark.parametrize("strided", [False, True])
def test_host_matrix_trains_the_same_trees(dp, orc, strided):
    """XGDMatrixCreateFromDense (host data, overlapped upload) grows the
    oracle's trees; with a row stride wider than the column count too."""
    rng = np.random.default_rng(31)
    R, F = 70000, 12  # several upload chunks
    x = rng.standard_normal((R, F)).astype(np.float32)
    x[rng.random((R, F)) < 0.05] = np.nan
    y = (np.nan_to_num(x[:, 0]) - 0.5 * np.nan_to_num(x[:, 3]) + 0.1 * rng.standard_normal(R)).astype(np.float32)
    xs = x
    if strided:
        wide = np.zeros((R, F + 5), np.float32)
        wide[:, :F] = x
        xs = wide[:, :F]
    params = {"objective": "reg:squarederror", "tree_method": "hist", "device": "cuda:0", "max_depth": 6,
              "max_bin": 256, "eta": 0.3}
    torch.cuda.set_device(0)
    d = dp.DMatrix.from_host(xs, y)
    assert d.num_row() == R and d.num_col() == F
    b = dp.train(params, d, 3)
    o = orc.Model(x, y, "reg:squarederror", max_depth=6, max_bin=256, eta=0.3, rounds=3, threads=8)
    compare_models(b, o, 1)
    np.testing.assert_array_equal(b.margins(R, 1).view(np.uint32), o.margins().view(np.uint32))


def test_host_matrix_refuses_inf_and_device_memory(dp):
    x = np.zeros((100, 3), np.float32)
    x[7, 1] = np.inf
    with pytest.raises(dp.DPError, match="inf"):
        dp.DMatrix.from_host(x)
    xd = torch.zeros((10, 3), device="cuda")
    with pytest.raises(dp.DPError, match="host memory"):
        h = dp.C.c_void_p()
        dp.check(dp.lib().XGDMatrixCreateFromDense(dp.array_interface(xd.data_ptr(), [10, 3]).encode(), b"{}",
                                                   dp.C.byref(h)))


def test_config_reports_cuda_updater_and_model_reloads(dp, orc, tmp_path):
    x, y = c1_data(3000, seed=2)
    b, o, _ = run(dp, orc, x, y, "binary:logistic", 3, max_depth=3)
    cfg = b.save_config()
    assert cfg["learner"]["generic_param"]["device"] == "cuda:0"
    assert cfg["learner"]["gradient_booster"]["updater"][0]["name"] == "grow_gpu_hist"
    p = tmp_path / "model.json"
    b.save_model(str(p))
    raw = p.read_bytes()
    assert raw == b.save_raw()
    c = dp.Booster()
    c.load_model(str(p))
    assert c.save_raw() == raw
    s = b.slice(0, 2)
    assert s.boosted_rounds() == 2 and s.trees() == b.trees()[:2]


def test_bad_labels_and_inf_are_refused(dp):
    x = np.zeros((10, 2), np.float32)
    y = np.full(10, 2.0, np.float32)
    d = dp.DMatrix.from_torch(cuda(x), cuda(y))
    b = dp.Booster({"objective": "binary:logistic"})
    with pytest.raises(dp.DPError, match="label"):
        b.update(d, 0)
    x[3, 1] = np.inf
    with pytest.raises(dp.DPError, match="inf"):
        dp.DMatrix.from_torch(cuda(x), cuda(y))


GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("name", sorted(p.stem for p in GOLDEN.glob("*.json")))
def test_golden_fixtures(dp, name):
    """The CUDA path against the independent restatement's fixtures."""
    d = json.loads((GOLDEN / f"{name}.json").read_text())
    x = np.array([[np.nan if v is None else v for v in r] for r in d["x"]], np.float32)
    y = np.array(d["y"], np.float32)
    p = d["params"]
    params = {"objective": d["objective"], "max_depth": p["max_depth"], "max_bin": p["max_bin"], "eta": p["eta"],
              "lambda": p["lambda"], "alpha": p["alpha"], "gamma": p["gamma"], "min_child_weight": p["mcw"]}
    if d["objective"].startswith("multi:"):
        params["num_class"] = d["num_class"]
    b = dp.train(params, dp.DMatrix.from_torch(cuda(x), cuda(y)), d["rounds"])
    trees = b.trees()
    assert len(trees) == len(d["expected"]["trees"])
    for t, e in zip(trees, d["expected"]["trees"]):
        assert t["left_children"] == e["left"] and t["right_children"] == e["right"]
        assert t["split_indices"] == e["feature"] and [int(v) for v in t["default_left"]] == e["dleft"]
        np.testing.assert_array_equal(np.array(t["split_conditions"], np.float32).view(np.uint32),
                                      np.array(e["cond"], np.float32).view(np.uint32))
    K = d["num_class"]
    np.testing.assert_array_equal(b.margins(len(y), K).view(np.uint32),
                                  np.array(d["expected"]["margin"], np.float32).view(np.uint32))


FROZEN = json.loads((GOLDEN / "configs" / "frozen.json").read_text())


@pytest.mark.parametrize("name", sorted(FROZEN))
def test_config_fixtures(dp, name):
    """Configs 1-4 (config 1 full size, the others scaled down) through the C
    API: the trees and training margins equal the frozen oracle outputs of
    tests/golden/make_config_fixtures.py bit for bit."""
    import sys
    sys.path.insert(0, str(GOLDEN))
    import config_data
    fx = FROZEN[name]
    x, y = config_data.data(name)
    params = {"objective": fx["objective"], "tree_method": "hist", "device": "cuda:0",
              "max_depth": fx["max_depth"], "max_bin": fx["max_bin"], "eta": fx["eta"]}
    if fx["objective"].startswith("multi:"):
        params["num_class"] = fx["num_class"]
    b = dp.train(params, dp.DMatrix.from_torch(cuda(x), cuda(y)), fx["rounds"])
    trees = b.trees()
    assert [len(t["left_children"]) for t in trees] == fx["nodes_per_tree"]
    assert config_data.tree_digest(trees) == fx["trees_sha256"]
    assert config_data.array_digest(b.margins(len(y), fx["num_class"])) == fx["margins_sha256"]
