"""The CPU oracle against an independent implementation of the same published
algorithm: scikit-learn's HistGradientBoosting (second-order boosting over
feature histograms, gain 0.5 (G_L^2/(H_L+l) + G_R^2/(H_R+l) - G^2/(H+l)),
leaf -G/(H+l) * eta, depth-limited growth, a learned direction for missing
values).  On integer features with at most 255 distinct values both give every
value its own bin, so the two grow the same trees; what separates them is the
oracle's fixed-point (g, h) quantiser (2^17 and 2^18 steps of each round's
largest |g| and h), which moves a margin by about 1e-6.

scikit-learn is not the parity oracle (its binning of general data, its
tie-breaking and its multiclass hessian differ), and XGBoost itself is absent:
this pins the oracle's gain, leaf, growth, missing-value and logistic
arithmetic to code written by others."""
import numpy as np
import pytest

sk = pytest.importorskip("sklearn.ensemble")


def data(seed, nan_frac, objective):
    rng = np.random.default_rng(seed)
    R, F = 20000, 6
    x = rng.integers(0, 32, (R, F)).astype(np.float32)
    sig = np.sin(x[:, 0] / 5) * 2 + (x[:, 1] > 15) * 1.5 - 0.05 * x[:, 2] * (x[:, 3] > 10)
    if nan_frac:
        x[rng.random((R, F)) < nan_frac] = np.nan
    if objective == "reg:squarederror":
        y = (sig + 0.1 * rng.standard_normal(R)).astype(np.float32)
    else:
        y = (sig + 0.5 * rng.standard_normal(R) > 0.8).astype(np.float32)
    return x, y


def splits_of_oracle(t):
    """(feature, boundary) of every internal node; the boundary is the
    smallest value routed right."""
    inner = np.array(t["left_children"]) >= 0
    return sorted(zip(np.array(t["split_indices"])[inner].tolist(),
                      np.array(t["split_conditions"], np.float64)[inner].tolist()))


def splits_of_sklearn(predictor):
    """(feature, boundary) of every internal node: scikit-learn stores the
    midpoint below the smallest value routed right, which on consecutive
    integers is that value - 0.5."""
    nodes = predictor.nodes
    inner = ~nodes["is_leaf"].astype(bool)
    return sorted(zip(nodes["feature_idx"][inner].tolist(), (nodes["num_threshold"][inner] + 0.5).tolist()))


@pytest.mark.parametrize("objective", ["reg:squarederror", "binary:logistic"])
@pytest.mark.parametrize("nan_frac", [0.0, 0.1])
@pytest.mark.parametrize("depth,seed", [(4, 2), (6, 3)])
def test_oracle_grows_the_trees_of_sklearn_histogram_boosting(orc, objective, nan_frac, depth, seed):
    x, y = data(seed, nan_frac, objective)
    rounds = 3
    common = dict(max_iter=rounds, max_depth=depth, max_leaf_nodes=None, learning_rate=0.3, l2_regularization=1.0,
                  min_samples_leaf=1, early_stopping=False, max_bins=255)
    if objective == "reg:squarederror":
        ref = sk.HistGradientBoostingRegressor(**common).fit(x, y)
        want = ref.predict(x)
        base = float(np.float32(y.astype(np.float64).mean()))   # scikit-learn starts from the mean
    else:
        ref = sk.HistGradientBoostingClassifier(**common).fit(x, y)
        want = ref.decision_function(x)
        p = y.astype(np.float64).mean()
        base = float(np.float32(np.log(p / (1 - p))))            # and from the log-odds
    m = orc.Model(x, y, objective, max_depth=depth, eta=0.3, reg_lambda=1.0, min_child_weight=0.0,
                  base_margin=base, rounds=rounds, threads=4)
    got = m.margins().reshape(-1).astype(np.float64)
    # measured: at most 2.4e-6 (squared error) and 1e-5 (logistic) on margins of about 2
    assert np.abs(got - want).max() < 1e-4
    predictors = getattr(ref, "_predictors", None)
    if predictors is None:  # the tree layout is scikit-learn's internal one
        return
    assert len(predictors) == m.num_trees() == rounds
    for i in range(rounds):
        mine, theirs = splits_of_oracle(m.tree(i)), splits_of_sklearn(predictors[i][0])
        if nan_frac:
            # with missing values, splits that route every training row alike
            # can be written differently (scikit-learn may split off the
            # missing values alone at an infinite threshold): compare the
            # features split on
            mine, theirs = sorted(f for f, _ in mine), sorted(f for f, _ in theirs)
        assert mine == theirs, i


@pytest.mark.parametrize("seed,nan_frac,depth", [(2, 0.0, 4), (3, 0.1, 5)])
def test_oracle_softprob_matches_sklearn_multiclass(orc, seed, nan_frac, depth):
    """multi:softprob takes the hessian 2 p (1 - p) (XGBoost's convention),
    scikit-learn p (1 - p).  With lambda = 0 that scales every gain of a node
    alike, so the splits are the same, and twice scikit-learn's learning rate
    gives the same leaves.  Exactly balanced classes make both start from
    uniform probabilities.  A split that scikit-learn takes at a gain that is
    zero up to rounding (the oracle's integer sums give exactly zero, and it
    does not split) changes no prediction, so the probabilities are compared."""
    rng = np.random.default_rng(seed)
    R, F, K = 21000, 6, 3
    x = rng.integers(0, 32, (R, F)).astype(np.float32)
    sig = np.sin(x[:, 0] / 5) * 2 + (x[:, 1] > 15) * 1.5 - 0.05 * x[:, 2] * (x[:, 3] > 10) + 0.3 * rng.standard_normal(R)
    y = np.empty(R, np.float32)
    y[np.argsort(sig, kind="stable")] = np.repeat(np.arange(K), R // K)
    if nan_frac:
        x[rng.random((R, F)) < nan_frac] = np.nan
    ref = sk.HistGradientBoostingClassifier(max_iter=3, max_depth=depth, max_leaf_nodes=None, learning_rate=0.3,
                                            l2_regularization=0.0, min_samples_leaf=1, early_stopping=False,
                                            max_bins=255).fit(x, y)
    m = orc.Model(x, y, "multi:softprob", num_class=K, max_depth=depth, eta=0.6, reg_lambda=0.0, min_child_weight=0.0,
                  rounds=3, threads=4)
    z = m.margins().reshape(R, K).astype(np.float64)
    p = np.exp(z - z.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    # measured: at most 2.1e-6
    assert np.abs(p - ref.predict_proba(x)).max() < 1e-4
