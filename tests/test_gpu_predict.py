"""XGBoosterPredictFromCudaArray (the call at native/class_study_train.cu:158
and native/class_model_native_adapter.cuh:30) against the oracle's
prediction: margins, objective outputs, round ranges, missing values, shapes.
Predicting the training matrix must reproduce the training margins bit for bit
(same leaves, added in the same order)."""
import json

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def data(R, F, seed, nan_frac=0.0):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((R, F)).astype(np.float32)
    if nan_frac:
        x[rng.random((R, F)) < nan_frac] = np.nan
    return x, rng


def train(dp, orc, x, y, objective, rounds, K=1, max_depth=5):
    params = {"objective": objective, "tree_method": "hist", "device": "cuda:0", "max_depth": max_depth,
              "max_bin": 256, "eta": 0.3}
    if objective.startswith("multi:"):
        params["num_class"] = K
    d = dp.DMatrix.from_torch(cuda(x), cuda(y))
    b = dp.train(params, d, rounds)
    o = orc.Model(x, y, objective, num_class=K, max_depth=max_depth, max_bin=256, eta=0.3, rounds=rounds, threads=8)
    return b, o, d


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.mark.parametrize("objective,K", [("reg:squarederror", 1), ("binary:logistic", 1), ("multi:softprob", 4),
                                         ("multi:softmax", 3)])
def test_prediction_matches_oracle(dp, orc, objective, K):
    x, rng = data(9000, 12, 40 + K, nan_frac=0.05)
    s = np.nan_to_num(x[:, 0]) + 0.5 * np.nan_to_num(x[:, 1])
    if objective == "binary:logistic":
        y = (s > 0).astype(np.float32)
    elif K > 1:
        y = np.digitize(s, np.linspace(-1, 1, K - 1)).astype(np.float32)
    else:
        y = (s + 0.1 * rng.standard_normal(len(s))).astype(np.float32)
    b, o, d = train(dp, orc, x, y, objective, 4, K)
    # training matrix: margins equal the training margins
    m = b.predict(cuda(x), margin=True).cpu().numpy()
    assert m.shape == (len(y), K)
    np.testing.assert_array_equal(bits(m), bits(b.margins(len(y), K)))
    # fresh rows with missing values, both output types, a round range
    xt, _ = data(5000, 12, 99, nan_frac=0.1)
    xt[:7, 3] = np.nan
    for margin in (True, False):
        got = b.predict(cuda(xt), margin=margin).cpu().numpy()
        want = o.predict(xt, margin=margin, objective=objective)
        assert got.shape == want.shape
        np.testing.assert_array_equal(bits(got), bits(want))
    got = b.predict(cuda(xt), margin=True, iteration_begin=1, iteration_end=3).cpu().numpy()
    np.testing.assert_array_equal(bits(got), bits(o.predict(xt, margin=True, iteration_begin=1, iteration_end=3)))


def test_prediction_shapes_and_reference_config(dp, orc):
    x, rng = data(3000, 6, 5)
    y = (x[:, 0] > 0).astype(np.float32)
    b, o, d = train(dp, orc, x, y, "binary:logistic", 3)
    assert tuple(b.predict(cuda(x), strict_shape=False).shape) == (3000,)
    assert tuple(b.predict(cuda(x), strict_shape=True).shape) == (3000, 1)
    # the exact configuration string the reference builds (class_study_train.cu:155-156)
    C = dp.C
    xt = cuda(x)
    cfg = json.dumps({"type": 0, "training": False, "iteration_begin": 0, "iteration_end": 0, "strict_shape": True,
                      "cache_id": 0})[:-1] + ',"missing":NaN}'
    shape = C.POINTER(C.c_uint64)()
    dims = C.c_uint64()
    out = C.POINTER(C.c_float)()
    dp.check(dp.lib().XGBoosterPredictFromCudaArray(b.handle, dp.array_interface(xt.data_ptr(), [3000, 6]).encode(),
                                                    cfg.encode(), None, C.byref(shape), C.byref(dims),
                                                    C.byref(out)))
    assert dims.value == 2 and shape[0] == 3000 and shape[1] == 1
    from cuda.bindings import runtime as rt
    err, attr = rt.cudaPointerGetAttributes(C.cast(out, C.c_void_p).value)
    assert attr.type == rt.cudaMemoryType.cudaMemoryTypeDevice and attr.device == 0


def test_prediction_after_reload_and_slice_and_strides(dp, orc):
    x, rng = data(6000, 10, 8, nan_frac=0.05)
    y = (np.nan_to_num(x[:, 2]) - np.nan_to_num(x[:, 5]) + 0.1 * rng.standard_normal(6000)).astype(np.float32)
    b, o, d = train(dp, orc, x, y, "reg:squarederror", 5)
    want = o.predict(x, margin=True)
    b2 = dp.Booster({"device": "cuda:0"}, [])
    b2.load_raw(b.save_raw())
    np.testing.assert_array_equal(bits(b2.predict(cuda(x), margin=True).cpu().numpy()), bits(want))
    s = b.slice(0, 2)
    np.testing.assert_array_equal(bits(s.predict(cuda(x), margin=True).cpu().numpy()),
                                  bits(o.predict(x, margin=True, iteration_end=2)))
    wide = np.zeros((6000, 16), np.float32)
    wide[:, :10] = x
    xs = cuda(wide)[:, :10]
    np.testing.assert_array_equal(bits(b.predict(xs, margin=True).cpu().numpy()), bits(want))


def test_prediction_errors(dp, orc):
    x, rng = data(2000, 6, 9)
    y = x[:, 0].copy()
    b, o, d = train(dp, orc, x, y, "reg:squarederror", 2)
    with pytest.raises(dp.DPError, match="num_feature"):
        b.predict(cuda(x[:, :2]))
    with pytest.raises(dp.DPError, match="iteration range"):
        b.predict(cuda(x), iteration_begin=1, iteration_end=5)
