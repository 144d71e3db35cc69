"""Host-side checks of the C-ABI library (no GPU): symbols, version contract,
parameter validation and the JSON model / configuration documents the
reference's callers read (native/class_model_native_adapter.cuh:24,
native/class_model_train.cu:48-51, native/class_io.hpp:131-205)."""
import json
import pathlib
import re

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]


def declared_symbols():
    text = (ROOT / "include" / "dp_gbdt.h").read_text()
    return re.findall(r"DP_API\s+[\w\s\*]+?\b(\w+)\s*\(", text)


def test_header_declares_the_reference_subset():
    names = set(declared_symbols())
    # every symbol the reference dlsym's on the training path
    # (native/class_native_training.cuh:51-69, native/class_model_native_adapter.cuh:21-30)
    for s in ["XGBoostVersion", "XGBuildInfo", "XGBGetLastError", "XGDMatrixCreateFromCudaArrayInterface",
              "XGDMatrixSetInfoFromInterface", "XGBoosterCreate", "XGBoosterSetParam", "XGBoosterUpdateOneIter",
              "XGBoosterSaveJsonConfig", "XGBoosterBoostedRounds", "XGBoosterSaveModel",
              "XGBoosterSaveModelToBuffer", "XGBoosterFree", "XGDMatrixFree", "XGBoosterLoadModelFromBuffer",
              "XGBoosterSlice", "XGBoosterLoadModel", "XGBoosterGetNumFeature"]:
        assert s in names


def test_library_exports_every_declared_symbol(dp):
    lib = dp.lib()
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing
    assert set(dp.EXPORTED) == set(declared_symbols())


def test_version_and_build_info(dp):
    assert dp.version() == (3, 4, 1)
    info = dp.build_info()
    assert info["USE_CUDA"] is True and info["DP_B200_GBDT"] is True


def test_parameters_follow_the_reference_tokens(dp):
    b = dp.Booster()
    # exactly the (key, token) pairs native/class_native_training.cuh:59-65 sends
    for k, v in {"objective": "multi:softmax", "num_class": "3", "tree_method": "hist", "device": "cuda:0",
                 "booster": "gbtree", "max_bin": "256", "max_depth": "6", "eta": "0.3", "lambda": "1.0",
                 "alpha": "0.0", "gamma": "0.0", "min_child_weight": "1.0", "subsample": "1",
                 "colsample_bytree": "1", "colsample_bylevel": "1", "colsample_bynode": "1",
                 "base_score": "[0,0,0]", "boost_from_average": "0", "seed": "0", "seed_per_iteration": "0",
                 "nthread": "2", "verbosity": "0", "validate_parameters": "1"}.items():
        b.set_param(k, v)
    cfg = b.save_config()
    assert cfg["learner"]["generic_param"]["device"] == "cuda:0"
    assert cfg["learner"]["gradient_booster"]["updater"][0]["name"] == "grow_gpu_hist"
    assert cfg["learner"]["objective"]["name"] == "multi:softmax"
    assert cfg["learner"]["learner_model_param"]["num_class"] == "3"
    assert cfg["dp_b200_gbdt"]["quantiser"] == {"grad_bits": 17, "hess_bits": 18, "window_rows": 16383}
    assert b.boosted_rounds() == 0


@pytest.mark.parametrize("key,value", [
    ("objective", "rank:pairwise"), ("max_depth", "0"), ("max_bin", "1"), ("eta", "-0.1"), ("lambda", "nan"),
    ("subsample", "0"), ("subsample", "1.5"), ("device", "cpu"), ("tree_method", "exact"), ("booster", "dart"),
    ("num_class", "-1"), ("max_depth", "2.5"),
])
def test_invalid_parameters_are_refused(dp, key, value):
    b = dp.Booster()
    with pytest.raises(dp.DPError):
        b.set_param(key, value)
    assert dp.lib().XGBGetLastError()


def test_null_handles_are_refused(dp):
    import ctypes as C
    n = C.c_int()
    assert dp.lib().XGBoosterBoostedRounds(None, C.byref(n)) == -1
    assert b"null" in dp.lib().XGBGetLastError()
    assert dp.lib().XGBoosterUpdateOneIter(None, 0, None) == -1
    assert dp.lib().dp_comm_set_timeout(None, 1000) == -1
    assert b"null" in dp.lib().XGBGetLastError()


def _model(objective="multi:softprob", K=2):
    return {
        "version": [3, 4, 1],
        "learner": {
            "learner_model_param": {"num_feature": "2", "num_class": str(K), "num_target": "1",
                                    "base_score": "[0,0]"},
            "objective": {"name": objective},
            "gradient_booster": {"name": "gbtree", "model": {
                "gbtree_model_param": {"num_trees": "2"}, "tree_info": [0, 1], "iteration_indptr": [0, 2],
                "trees": [{"id": i, "tree_param": {"num_nodes": "3", "size_leaf_vector": "1"}, "categories": [],
                           "split_type": [0, 0, 0], "left_children": [1, -1, -1], "right_children": [2, -1, -1],
                           "split_indices": [i, 0, 0], "split_conditions": [0.5, -1.0, 0.1 + i],
                           "default_left": [True, False, False]} for i in range(2)]}}}}


def test_model_buffer_round_trip_and_slice(dp):
    b = dp.Booster()
    b.load_raw(json.dumps(_model()).encode())
    assert b.boosted_rounds() == 1 and b.num_features() == 2
    doc = json.loads(b.save_raw())
    assert doc["version"] == [3, 4, 1]
    lr = doc["learner"]
    assert lr["objective"]["name"] == "multi:softprob"
    assert lr["learner_model_param"]["num_class"] == "2" and lr["learner_model_param"]["num_feature"] == "2"
    trees = lr["gradient_booster"]["model"]["trees"]
    assert [t["split_conditions"] for t in trees] == [[0.5, -1.0, 0.1], [0.5, -1.0, 1.1]]
    for t in trees:
        for i, (l, r) in enumerate(zip(t["left_children"], t["right_children"])):
            assert (l == -1 and r == -1) or (l > i and r == l + 1)  # native/class_native_source_contract.hpp:26-33
    s = b.slice(0, 1)
    assert s.boosted_rounds() == 1
    assert json.loads(s.save_raw())["learner"]["gradient_booster"]["model"]["tree_info"] == [0, 1]


def test_float_format_round_trips_through_double(dp, tmp_path):
    import numpy as np
    rng = np.random.default_rng(7)
    vals = np.concatenate([rng.standard_normal(2000).astype(np.float32),
                           np.array([1e-38, 3.4028235e38, -0.0, 0.0, 0.1, 1 / 3], np.float32)])
    m = _model()
    m["learner"]["gradient_booster"]["model"]["trees"][0]["split_conditions"] = [float(vals[0]), -1.0, 1.0]
    b = dp.Booster()
    for v in vals:
        m["learner"]["gradient_booster"]["model"]["trees"][0]["split_conditions"][0] = float(v)
        b.load_raw(json.dumps(m).encode())
        out = json.loads(b.save_raw())["learner"]["gradient_booster"]["model"]["trees"][0]["split_conditions"][0]
        # double parse then narrow, as native/class_io.hpp:180 does; the sign of zero survives
        assert np.float32(out).view(np.uint32) == v.view(np.uint32)


def test_release_cached_memory_with_nothing_kept(dp):
    # nothing has been freed in this process: no allocation is kept, and the
    # call succeeds without touching a device
    assert dp.lib().dp_release_cached_memory() == 0
