"""CPU checks of the oracle (test infrastructure): hand-computed known answers
and the golden fixtures produced by tests/golden/make_golden.py, an
independent pure-Python restatement of the same rules.  XGBoost 3.4.1 (where
the reference's arithmetic lives) is absent, so these pin the oracle to its
written semantics, not to XGBoost."""
import json
import math
import pathlib

import numpy as np
import pytest

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"
CASES = sorted(p.stem for p in GOLDEN.glob("*.json"))


def load_case(name):
    d = json.loads((GOLDEN / f"{name}.json").read_text())
    x = np.array([[np.nan if v is None else v for v in r] for r in d["x"]], np.float32)
    return d, x, np.array(d["y"], np.float32)


def test_exp_is_accurate(orc):
    xs = np.concatenate([np.linspace(-700, 700, 20001), np.linspace(-2, 2, 20001), [0.0, 1e-300, -1e-300]])
    for x in xs:
        e = orc.dp_exp(float(x))
        ref = math.exp(x)
        assert abs(e - ref) <= 4e-16 * ref, (x, e, ref)
    assert orc.dp_exp(710.0) == math.inf and orc.dp_exp(-800.0) == 0.0


def test_hand_computed_stump(orc):
    # x = 1..4, y = 1,1,3,3, squared error, lambda 0, eta 1, mcw 0: g = -y, h = 1.
    # Candidates (x < 2, 3, 4) give gains 2/3, 2, 2/3 -> split x < 3, leaves 1 and 3.
    x = np.array([[1.0], [2.0], [3.0], [4.0]], np.float32)
    y = np.array([1, 1, 3, 3], np.float32)
    m = orc.Model(x, y, "reg:squarederror", max_depth=1, eta=1.0, reg_lambda=0.0, min_child_weight=0.0, rounds=1)
    t = m.tree(0)
    assert t["left_children"].tolist() == [1, -1, -1] and t["right_children"].tolist() == [2, -1, -1]
    assert t["split_conditions"].tolist() == [3.0, 1.0, 3.0]
    assert t["loss_changes"][0] == np.float32(2.0)
    assert t["sum_hessian"].tolist() == [4.0, 2.0, 2.0]
    np.testing.assert_array_equal(m.margins()[:, 0], [1, 1, 3, 3])


@pytest.mark.parametrize("y,params,split,gain,leaves", [
    # alpha 1: T(G) = sign(G) max(|G| - 1, 0).  Parent G = -8, H = 4: s = 49/4.
    # x < 3: s_L = 1/2, s_R = 25/2 -> gain 0.375 (x < 2: -0.125, x < 4: -1.458);
    # leaves -T(G)/H = 0.5 and 2.5
    ([1, 1, 3, 3], {"alpha": 1.0}, 3.0, 0.375, (0.5, 2.5)),
    # gamma 1.5 comes off the best gain 2 (x < 3): 0.5 > 0, so the split stays
    ([1, 1, 3, 3], {"gamma": 1.5}, 3.0, 0.5, (1.0, 3.0)),
    # gamma 2.5 leaves no positive gain: the root is a leaf, -G/H = 8/4
    ([1, 1, 3, 3], {"gamma": 2.5}, None, None, (2.0,)),
    # min_child_weight 2.5: every candidate has a side with H < 2.5
    ([1, 1, 3, 3], {"min_child_weight": 2.5}, None, None, (2.0,)),
    # y = 0, 4, 4, 4: the best split x < 2 (gain 6) has H_L = 1; with
    # min_child_weight 1.5 only x < 3 is valid (gain 0.5 (8 + 32 - 36) = 2)
    ([0, 4, 4, 4], {"min_child_weight": 1.5}, 3.0, 2.0, (2.0, 4.0)),
])
def test_regularisation_by_hand(orc, y, params, split, gain, leaves):
    # x = 1..4, squared error from margin 0 (g = -y, h = 1), lambda 0, eta 1;
    # the quantiser scales are powers of two, so every sum here is exact
    x = np.array([[1.0], [2.0], [3.0], [4.0]], np.float32)
    kw = {"reg_lambda": 0.0, "min_child_weight": 0.0} | params
    m = orc.Model(x, np.array(y, np.float32), "reg:squarederror", max_depth=1, eta=1.0, rounds=1, **kw)
    t = m.tree(0)
    if split is None:
        assert t["left_children"].tolist() == [-1]
        assert t["split_conditions"].tolist() == list(leaves)
        np.testing.assert_array_equal(m.margins()[:, 0], [leaves[0]] * 4)
    else:
        assert t["left_children"].tolist() == [1, -1, -1] and t["right_children"].tolist() == [2, -1, -1]
        assert t["split_conditions"].tolist() == [split, *leaves]
        assert t["loss_changes"][0] == np.float32(gain)
        np.testing.assert_array_equal(m.margins()[:, 0], [leaves[0], leaves[0], leaves[1], leaves[1]])


def test_logistic_stump_by_hand(orc):
    # margin 0: p = 1/2, g = 1/2 - y, h = 1/4.  y = 0, 0, 1, 1, lambda 0: parent
    # G = 0 (s = 0); x < 3 has G = +-1, H = 1/2 on each side: gain 0.5 (2 + 2) = 2
    # (x < 2 and x < 4: 2/3); leaves -G/H = -2 and 2
    x = np.array([[1.0], [2.0], [3.0], [4.0]], np.float32)
    m = orc.Model(x, np.array([0, 0, 1, 1], np.float32), "binary:logistic", max_depth=1, eta=1.0, reg_lambda=0.0,
                  min_child_weight=0.0, rounds=1)
    t = m.tree(0)
    assert t["split_conditions"].tolist() == [3.0, -2.0, 2.0]
    assert t["loss_changes"][0] == np.float32(2.0)
    assert t["sum_hessian"].tolist() == [1.0, 0.5, 0.5]
    np.testing.assert_array_equal(m.margins()[:, 0], [-2, -2, 2, 2])


def test_softprob_stumps_by_hand(orc):
    # two classes from margin 0: p_k = 1/2, g_k = 1/2 - [y = k], h_k = 2 p (1 - p)
    # = 1/2.  y = 0, 0, 1, 1, lambda 0: in each class's tree x < 3 has G = +-1,
    # H = 1 on each side and parent G = 0: gain 0.5 (1 + 1) = 1; leaves -G/H
    x = np.array([[1.0], [2.0], [3.0], [4.0]], np.float32)
    m = orc.Model(x, np.array([0, 0, 1, 1], np.float32), "multi:softprob", num_class=2, max_depth=1, eta=1.0,
                  reg_lambda=0.0, min_child_weight=0.0, rounds=1)
    assert m.num_trees() == 2
    assert m.tree(0)["split_conditions"].tolist() == [3.0, 1.0, -1.0]
    assert m.tree(1)["split_conditions"].tolist() == [3.0, -1.0, 1.0]
    for k in range(2):
        assert m.tree(k)["loss_changes"][0] == np.float32(1.0)
    np.testing.assert_array_equal(m.margins(), [[1, -1], [1, -1], [-1, 1], [-1, 1]])


@pytest.mark.parametrize("y,gain,default_left,leaves,margins", [
    # x = 1, 2, 3, NaN (bins 0, 1, 2 and the missing code), lambda 0.
    # y = 1, 1, 3, 3: parent G = -8, H = 4 (s = 16).  x < 3 with the missing row
    # right: s_L = 4/2, s_R = 36/2 -> gain 2; left: 25/3 + 9 -> 0.667; x < 2:
    # 0.667 (right) and 0 (left).  Missing goes right; leaves 1 and 3
    ([1, 1, 3, 3], 2.0, 0, (1.0, 3.0), [1, 1, 3, 3]),
    # y = 1, 1, 3, 1: parent G = -6 (s = 9).  x < 3 with the missing row left:
    # s_L = 9/3, s_R = 9/1 -> gain 1.5; right: 0.5; x < 2: 0.5 (left), 0.167
    # (right).  Missing goes left; leaves 1 and 3, and the NaN row gets 1
    ([1, 1, 3, 1], 1.5, 1, (1.0, 3.0), [1, 1, 3, 1]),
])
def test_missing_value_direction_by_hand(orc, y, gain, default_left, leaves, margins):
    x = np.array([[1.0], [2.0], [3.0], [np.nan]], np.float32)
    m = orc.Model(x, np.array(y, np.float32), "reg:squarederror", max_depth=1, eta=1.0, reg_lambda=0.0,
                  min_child_weight=0.0, rounds=1)
    t = m.tree(0)
    assert t["split_conditions"].tolist() == [3.0, *leaves]
    assert t["default_left"][0] == default_left
    assert t["loss_changes"][0] == np.float32(gain)
    np.testing.assert_array_equal(m.margins()[:, 0], margins)


def test_depth_two_tree_by_hand(orc):
    # y = 1..4, lambda 0: root x < 3 (gain 0.5 (4.5 + 24.5 - 25) = 2; x < 2 and
    # x < 4 give 1.5); then x < 2 under node 1 and x < 4 under node 2, each
    # 0.25 (the other bins leave a side with H = 0, which is not valid).  Nodes
    # are numbered in creation order: 1, 2 the root's children, 3..6 theirs
    x = np.array([[1.0], [2.0], [3.0], [4.0]], np.float32)
    m = orc.Model(x, np.array([1, 2, 3, 4], np.float32), "reg:squarederror", max_depth=2, eta=1.0, reg_lambda=0.0,
                  min_child_weight=0.0, rounds=1)
    t = m.tree(0)
    assert t["left_children"].tolist() == [1, 3, 5, -1, -1, -1, -1]
    assert t["right_children"].tolist() == [2, 4, 6, -1, -1, -1, -1]
    assert t["split_conditions"].tolist() == [3.0, 2.0, 4.0, 1.0, 2.0, 3.0, 4.0]
    assert t["loss_changes"][:3].tolist() == [2.0, 0.25, 0.25]
    np.testing.assert_array_equal(m.margins()[:, 0], [1, 2, 3, 4])


def test_second_round_by_hand(orc):
    # eta 0.5, lambda 0, y = 1, 1, 3, 3.  Round 1: x < 3, leaves 0.5 and 1.5.
    # Round 2 from those margins: g = -0.5, -0.5, -1.5, -1.5, parent G = -4
    # (s = 4); x < 3: 0.5 (1/2 + 9/2 - 4) = 0.5, the others 1/6; leaves
    # 0.5 * (1/2) = 0.25 and 0.5 * (3/2) = 0.75
    x = np.array([[1.0], [2.0], [3.0], [4.0]], np.float32)
    m = orc.Model(x, np.array([1, 1, 3, 3], np.float32), "reg:squarederror", max_depth=1, eta=0.5, reg_lambda=0.0,
                  min_child_weight=0.0, rounds=2)
    assert m.tree(0)["split_conditions"].tolist() == [3.0, 0.5, 1.5]
    assert m.tree(1)["split_conditions"].tolist() == [3.0, 0.25, 0.75]
    assert m.tree(1)["loss_changes"][0] == np.float32(0.5)
    np.testing.assert_array_equal(m.margins()[:, 0], [0.75, 0.75, 2.25, 2.25])


def test_quantile_boundaries_by_hand(orc):
    # 10 distinct values, max_bin 4: ranks floor(k*10/4) = 2, 5, 7 -> values 20, 50, 70
    x = (np.arange(10, dtype=np.float32) * 10)[::-1].reshape(-1, 1).copy()
    cut, nb, hm = orc.cuts(x, 4)
    assert nb[0] == 4 and hm[0] == 0
    assert cut[0, :3].tolist() == [20.0, 50.0, 70.0]
    bins = orc.bin_matrix(x, cut, nb, hm)[:, 0]
    assert bins[::-1].tolist() == [0, 0, 1, 1, 1, 2, 2, 3, 3, 3]


@pytest.mark.parametrize("values,max_bin,bounds,bins", [
    # 4 distinct values, max_bin 4: every distinct value but the minimum
    ([1, 1, 1, 1, 2, 2, 3, 4], 4, [2, 3, 4], [0, 0, 0, 0, 1, 1, 2, 3]),
    # 7 distinct > 3: ranks floor(k 10 / 3) = 3, 6 -> values 3, 4
    ([1, 2, 3, 3, 3, 3, 4, 5, 6, 7], 3, [3, 4], [0, 0, 1, 1, 1, 1, 2, 2, 2, 2]),
    # ranks 3 and 6 both hold 5: one boundary after deduplication
    ([1, 5, 5, 5, 5, 5, 5, 5, 7, 9], 3, [5], [0, 1, 1, 1, 1, 1, 1, 1, 1, 1]),
    # ranks 3 and 6 hold the minimum, which is never a boundary: one bin
    ([1, 1, 1, 1, 1, 1, 1, 2, 3, 4], 3, [], [0] * 10),
])
def test_cut_ranks_and_duplicates_by_hand(orc, values, max_bin, bounds, bins):
    x = np.array(values, np.float32)[::-1].reshape(-1, 1).copy()  # order of the rows is irrelevant
    cut, nb, hm = orc.cuts(x, max_bin)
    assert hm[0] == 0 and nb[0] == len(bounds) + 1
    assert cut[0, :len(bounds)].tolist() == [float(v) for v in bounds]
    assert orc.bin_matrix(x, cut, nb, hm)[::-1, 0].tolist() == bins


def test_missing_values_take_the_reserved_code(orc):
    x = np.array([[np.nan], [1.0], [2.0], [-0.0], [0.0]], np.float32)
    cut, nb, hm = orc.cuts(x, 256)
    assert hm[0] == 1 and nb[0] == 3  # distinct {0, 1, 2}; -0.0 folds into 0.0
    assert cut[0, :2].tolist() == [1.0, 2.0]
    assert orc.bin_matrix(x, cut, nb, hm)[:, 0].tolist() == [255, 1, 2, 0, 0]


def test_quantiser_scale(orc):
    gh = np.array([[0.75, 0.25], [-3.0, 0.1]], np.float32)
    sg, sh = orc.quantizer(gh)
    assert sg == 2.0 ** 15 and sh == 2.0 ** 19  # |g| < 4 -> 2^(17-2); h < 0.5 -> 2^(18-(-1))
    assert orc.quantizer(np.zeros((3, 2), np.float32)) == (1.0, 1.0)


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_golden_restatement(orc, name):
    d, x, y = load_case(name)
    p = d["params"]
    exp = d["expected"]
    cut, nb, hm = orc.cuts(x, p["max_bin"])
    assert nb.tolist() == exp["nbins"] and hm.tolist() == exp["has_missing"]
    for f, b in enumerate(exp["bounds"]):
        np.testing.assert_array_equal(cut[f, : len(b)], np.array(b, np.float32))
    np.testing.assert_array_equal(orc.bin_matrix(x, cut, nb, hm)[:, : x.shape[1]], np.array(exp["bins"]))
    m = orc.Model(x, y, d["objective"], num_class=d["num_class"], max_depth=p["max_depth"], max_bin=p["max_bin"],
                  eta=p["eta"], reg_lambda=p["lambda"], alpha=p["alpha"], gamma=p["gamma"],
                  min_child_weight=p["mcw"], rounds=d["rounds"])
    assert m.num_trees() == len(exp["trees"])
    for i, t in enumerate(exp["trees"]):
        ot = m.tree(i)
        assert ot["left_children"].tolist() == t["left"]
        assert ot["right_children"].tolist() == t["right"]
        assert ot["split_indices"].tolist() == t["feature"]
        assert ot["default_left"].tolist() == t["dleft"]
        np.testing.assert_array_equal(ot["split_conditions"].view(np.uint32),
                                      np.array(t["cond"], np.float32).view(np.uint32))
    np.testing.assert_array_equal(m.margins().view(np.uint32), np.array(exp["margin"], np.float32).view(np.uint32))


def test_threads_and_subtraction_do_not_change_trees(orc):
    d, x, y = load_case("logistic_nan")
    rng = np.random.default_rng(3)
    x = rng.standard_normal((5000, 12)).astype(np.float32)
    x[rng.random(x.shape) < 0.1] = np.nan
    y = (np.nan_to_num(x[:, 0]) > 0).astype(np.float32)
    a = orc.Model(x, y, "binary:logistic", max_depth=6, rounds=3, threads=1, subtract=False)
    b = orc.Model(x, y, "binary:logistic", max_depth=6, rounds=3, threads=8, subtract=True)
    for i in range(3):
        for k, v in a.tree(i).items():
            np.testing.assert_array_equal(v, b.tree(i)[k])


def test_oracle_prediction_reproduces_training_margins(orc):
    """Prediction of the training rows adds the same leaves in the same order
    as training, so it returns the training margins bit for bit; the
    transforms follow the gradients' arithmetic."""
    rng = np.random.default_rng(17)
    x = rng.standard_normal((2500, 7)).astype(np.float32)
    x[rng.random(x.shape) < 0.1] = np.nan
    s = np.nan_to_num(x[:, 0]) - np.nan_to_num(x[:, 4])
    for objective, K, y in [("binary:logistic", 1, (s > 0).astype(np.float32)),
                            ("multi:softprob", 3, np.digitize(s, [-0.5, 0.5]).astype(np.float32)),
                            ("reg:squarederror", 1, s.astype(np.float32))]:
        m = orc.Model(x, y, objective, num_class=K, max_depth=4, rounds=4, threads=4)
        mg = m.predict(x, margin=True)
        np.testing.assert_array_equal(mg.view(np.uint32), m.margins().view(np.uint32))
        out = m.predict(x, objective=objective)
        if objective == "binary:logistic":
            np.testing.assert_allclose(out[:, 0], 1 / (1 + np.exp(-mg[:, 0].astype(np.float64))), rtol=1e-6)
        elif objective == "multi:softprob":
            e = np.exp(mg.astype(np.float64) - mg.max(1, keepdims=True))
            np.testing.assert_allclose(out, e / e.sum(1, keepdims=True), rtol=1e-6)
        else:
            np.testing.assert_array_equal(out, mg)
        # rounds [1, 3) = margins of the full model minus rounds 0 and 3 is not
        # float-exact, so compare against a fresh accumulation instead
        part = m.predict(x, margin=True, iteration_begin=1, iteration_end=3)
        assert part.shape == mg.shape and np.isfinite(part).all()


def test_oracle_prediction_routing_by_hand(orc):
    """A stump on feature 0: rows with x0 < cond go left, NaN follows
    default_left; leaf values come back as margins."""
    x = np.array([[0.0], [1.0], [2.0], [3.0]], np.float32)
    y = np.array([0.0, 0.0, 4.0, 4.0], np.float32)
    m = orc.Model(x, y, "reg:squarederror", max_depth=1, reg_lambda=0.0, min_child_weight=0.0, eta=1.0, rounds=1)
    t = m.tree(0)
    cond, dl = t["split_conditions"][0], t["default_left"][0]
    left, right = t["split_conditions"][t["left_children"][0]], t["split_conditions"][t["right_children"][0]]
    xt = np.array([[cond - 1e-3], [cond], [np.nan]], np.float32)
    got = m.predict(xt, margin=True)[:, 0]
    np.testing.assert_array_equal(got, np.array([left, right, left if dl else right], np.float32))


FROZEN = json.loads((GOLDEN / "configs" / "frozen.json").read_text())


@pytest.mark.parametrize("name", sorted(FROZEN))
def test_oracle_reproduces_config_fixtures(orc, name):
    """The oracle on configs 1-4 (config 1 full size, the others scaled down;
    tests/golden/config_data.py) still gives the frozen cuts, trees and margins
    of tests/golden/make_config_fixtures.py."""
    import hashlib
    import sys
    sys.path.insert(0, str(GOLDEN))
    import config_data
    fx = FROZEN[name]
    x, y = config_data.data(name)
    assert x.shape == (fx["rows"], fx["features"])
    m = orc.Model(x, y, fx["objective"], num_class=fx["num_class"], max_depth=fx["max_depth"],
                  max_bin=fx["max_bin"], eta=fx["eta"], rounds=fx["rounds"], threads=4)
    cut, nb, hm = m.cuts()
    hc = hashlib.sha256()
    for f in range(x.shape[1]):
        hc.update(np.asarray(cut[f][: max(int(nb[f]) - 1, 0)], dtype="<f4").tobytes())
    hc.update(np.asarray(nb, dtype="<u2").tobytes())
    hc.update(np.asarray(hm, dtype=np.uint8).tobytes())
    assert hc.hexdigest() == fx["cuts_sha256"]
    trees = [m.tree(i) for i in range(m.num_trees())]
    assert [len(t["left_children"]) for t in trees] == fx["nodes_per_tree"]
    assert config_data.tree_digest(trees) == fx["trees_sha256"]
    assert config_data.array_digest(m.margins()) == fx["margins_sha256"]
