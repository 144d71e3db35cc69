"""Drop-in check: the reference's own FIT-only trainer (native/class_model_train.cu,
compiled unmodified from the reference sources into oracle/_ref/) binds
libdp_gbdt.so through its plan's native_library_path, trains, and its own
checks pass: the CUDA updater and device (native/class_model_train.cu:48),
the completed round count (:49), the saved objective and shape (:50-51).  The
model it writes must equal the oracle's trees for the same inputs."""
import hashlib
import json
import pathlib
import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = pathlib.Path(__file__).resolve().parents[1]
TRAINER = ROOT / "oracle" / "_ref" / "class_model_train"
LIB = ROOT / "decision-programs_b200" / "libdp_gbdt.so"


def sha(p: pathlib.Path) -> str:
    return hashlib.sha256(p.read_bytes()).hexdigest()


@pytest.mark.skipif(not TRAINER.exists(), reason="reference trainer not built (needs the reference sources)")
def test_reference_trainer_runs_on_libdp_gbdt(orc, tmp_path):
    rng = np.random.default_rng(21)
    R, F, K = 3000, 6, 3
    x = rng.standard_normal((R, F)).astype(np.float32)
    x[rng.random((R, F)) < 0.05] = np.nan
    y = np.argmax(np.nan_to_num(x[:, :3]) + 0.3 * rng.standard_normal((R, 3)), 1).astype(np.uint32)
    values, labels = tmp_path / "values.fp32", tmp_path / "labels.u32"
    values.write_bytes(x.astype("<f4").tobytes())
    labels.write_bytes(y.astype("<u4").tobytes())
    manifest = json.loads(subprocess.run([str(TRAINER), "source-manifest"], check=True, capture_output=True,
                                         text=True).stdout)
    hp = {"rounds": 4, "max_depth": 3, "eta": 0.3, "max_bin": 256, "lambda": 1.0, "min_child_weight": 1.0}
    plan = {
        "format": "class-model-training-plan-1", "TEST_read": False, "VALID_read": False,
        "selection_performed": False, "training_performed": True,
        "dataset": {"format": "dense-fp32-u32-class-labels-1", "TEST_read": False, "features": F, "classes": K,
                    "rows": R, "row_stride": F, "FIT_rows": R, "VALID_rows": 0, "preprocessing": "seeded synthetic",
                    "values_path": str(values), "labels_path": str(labels), "values_sha256": sha(values),
                    "labels_sha256": sha(labels)},
        "hyperparameters": hp,
        "native_library_path": str(LIB), "native_library_sha256": sha(LIB),
        "executable_sha256": sha(TRAINER), "source_manifest_sha256": manifest["sha256"],
    }
    plan_path = tmp_path / "plan.json"
    plan_path.write_text(json.dumps(plan))
    out = tmp_path / "out"
    r = subprocess.run([str(TRAINER), "fit", str(plan_path), sha(plan_path), str(out)], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr + r.stdout
    result = json.loads((out / "result.json").read_text())
    assert result["complete"] and result["CUDA_executed"] and result["native_objective"] == "multi:softmax"
    cfg = json.loads((out / "configuration.json").read_text())
    assert cfg["learner"]["gradient_booster"]["updater"][0]["name"] == "grow_gpu_hist"
    model = json.loads((out / "model.json").read_text())
    trees = model["learner"]["gradient_booster"]["model"]["trees"]
    o = orc.Model(x, y.astype(np.float32), "multi:softmax", num_class=K, max_depth=3, max_bin=256, eta=0.3,
                  rounds=4, threads=4)
    assert len(trees) == o.num_trees() == 4 * K
    for i, t in enumerate(trees):
        ot = o.tree(i)
        for f in ["left_children", "right_children", "split_indices"]:
            np.testing.assert_array_equal(np.array(t[f]), ot[f])
        np.testing.assert_array_equal(np.array(t["default_left"], np.uint8), ot["default_left"])
        np.testing.assert_array_equal(np.array(t["split_conditions"], np.float32).view(np.uint32),
                                      ot["split_conditions"].view(np.uint32))


READER = ROOT / "oracle" / "_ref" / "ref_read_model"


@pytest.mark.skipif(not READER.exists(), reason="reference reader not built (needs the reference sources)")
def test_reference_converter_reads_gpu_trained_models(dp, orc, tmp_path):
    """A multi:softprob model trained on the GPU and saved through
    XGBoosterSaveModel is read by the reference converter's reader
    (native/class_io.hpp:99-242) with the oracle's trees bit for bit."""
    import torch
    from test_ref_reader import check_against_trees, read_with_reference

    rng = np.random.default_rng(33)
    R, F, K = 6000, 9, 5
    x = rng.standard_normal((R, F)).astype(np.float32)
    x[rng.random((R, F)) < 0.05] = np.nan
    y = np.argmax(np.nan_to_num(x[:, :K]) + 0.4 * rng.standard_normal((R, K)), 1).astype(np.float32)
    params = {"objective": "multi:softprob", "num_class": K, "tree_method": "hist", "device": "cuda:0",
              "max_depth": 4, "max_bin": 256, "eta": 0.3}
    d = dp.DMatrix.from_torch(torch.from_numpy(x).cuda(), torch.from_numpy(y).cuda())
    b = dp.train(params, d, 3)
    path = tmp_path / "model.json"
    b.save_model(str(path))
    doc = read_with_reference(path)
    o = orc.Model(x, y, "multi:softprob", num_class=K, max_depth=4, max_bin=256, eta=0.3, rounds=3, threads=8)
    trees = []
    for i in range(o.num_trees()):
        t = o.tree(i)
        t["klass"] = i % K
        trees.append(t)
    check_against_trees(doc, trees, K)
    assert doc["features"] == F


CONVERT = ROOT / "oracle" / "_ref" / "ref_convert_check"
LIBRARY = ROOT / "decision-programs_b200" / "libdp_gbdt.so"


@pytest.mark.skipif(not CONVERT.exists(), reason="reference converter harness not built (needs the reference sources)")
@pytest.mark.parametrize("objective", ["multi:softprob", "multi:softmax"])
def test_reference_converter_native_session(dp, orc, tmp_path, objective):
    """The reference converter's acceptance of a GPU-trained model, run by the
    converter's own code (native/class_model_convert.cpp, compiled unmodified):
    source_shape() gates the model JSON, then its ResidentModel dlopens
    libdp_gbdt as the native library, checks version and CUDA build, loads the
    model from its buffer, checks feature count, objective, classes and device
    in the JSON configuration, and predicts rows from device memory.  Its
    margins and outputs equal the oracle's predictions bit for bit."""
    import torch

    rng = np.random.default_rng(44)
    R, F, K = 5000, 7, 4
    x = rng.standard_normal((R, F)).astype(np.float32)
    x[rng.random((R, F)) < 0.05] = np.nan
    y = np.argmax(np.nan_to_num(x[:, :K]) + 0.5 * rng.standard_normal((R, K)), 1).astype(np.float32)
    params = {"objective": objective, "num_class": K, "tree_method": "hist", "device": "cuda:0",
              "max_depth": 4, "max_bin": 256, "eta": 0.3}
    d = dp.DMatrix.from_torch(torch.from_numpy(x).cuda(), torch.from_numpy(y).cuda())
    b = dp.train(params, d, 3)
    model = tmp_path / "model.json"
    b.save_model(str(model))
    rows = 700
    xr = np.ascontiguousarray(x[:rows])
    (tmp_path / "rows.f32").write_bytes(xr.tobytes())
    r = subprocess.run([str(CONVERT), "native", str(model), str(LIBRARY), str(tmp_path / "rows.f32"), str(rows)],
                       capture_output=True, text=True, timeout=300)
    doc = json.loads(r.stdout)
    assert r.returncode == 0 and doc["ok"], doc
    assert (doc["features"], doc["classes"], doc["objective"]) == (F, K, objective)
    o = orc.Model(x, y, objective, num_class=K, max_depth=4, max_bin=256, eta=0.3, rounds=3, threads=8)
    margins = np.asarray(doc["margin_bits"], np.uint32).view(np.float32).reshape(rows, K)
    np.testing.assert_array_equal(margins.view(np.uint32), o.predict(xr, margin=True).reshape(rows, K).view(np.uint32))
    out = np.asarray(doc["output_bits"], np.uint32).view(np.float32)
    np.testing.assert_array_equal(out.view(np.uint32), o.predict(xr).reshape(out.shape).view(np.uint32))


RESIDENT = ROOT / "oracle" / "_ref" / "ref_resident"


@pytest.mark.skipif(not RESIDENT.exists(), reason="reference resident trainer not built (needs the reference sources)")
def test_reference_resident_trainer_lifecycle(orc, tmp_path):
    """The reference's resident trainer (native/class_study_train.cu, built
    unmodified with the harness oracle/ref_resident.cpp) trains through
    libdp_gbdt.so, predicts classes, margins and probabilities from device
    memory, slices a round prefix (XGBoosterSlice) and restores the full model
    from its buffer (XGBoosterLoadModelFromBuffer); its own checks on shapes,
    device output, configuration and round counts run on every call.  Models
    and predictions must equal the oracle's bit for bit."""
    rng = np.random.default_rng(57)
    R, F, K, rounds, cut = 4000, 7, 4, 5, 2
    x = rng.standard_normal((R, F)).astype(np.float32)
    x[rng.random((R, F)) < 0.04] = np.nan
    y = np.argmax(np.nan_to_num(x[:, :K]) + 0.3 * rng.standard_normal((R, K)), 1).astype(np.uint32)
    (tmp_path / "values.f32").write_bytes(x.astype("<f4").tobytes())
    (tmp_path / "labels.u32").write_bytes(y.astype("<u4").tobytes())
    (tmp_path / "meta.json").write_text(json.dumps({"rows": R, "features": F, "classes": K, "rounds": rounds,
                                                    "max_depth": 4, "slice_rounds": cut}))
    r = subprocess.run([str(RESIDENT), str(LIB), sha(LIB), str(tmp_path)], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr + r.stdout

    def f32(name, shape):
        return np.fromfile(tmp_path / name, dtype="<f4").reshape(shape)

    o = orc.Model(x, y.astype(np.float32), "multi:softmax", num_class=K, max_depth=4, max_bin=256, eta=0.3,
                  rounds=rounds, threads=4)
    bits = lambda a: np.ascontiguousarray(a, np.float32).view(np.uint32)  # noqa: E731
    model = json.loads((tmp_path / "model.json").read_text())
    trees = model["learner"]["gradient_booster"]["model"]["trees"]
    assert len(trees) == o.num_trees() == rounds * K
    for i, t in enumerate(trees):
        ot = o.tree(i)
        for f in ["left_children", "right_children", "split_indices"]:
            np.testing.assert_array_equal(np.array(t[f]), ot[f])
        np.testing.assert_array_equal(bits(t["split_conditions"]), bits(ot["split_conditions"]))
    margins = o.predict(x, margin=True)
    np.testing.assert_array_equal(bits(f32("margins.f32", (R, K))), bits(margins))
    np.testing.assert_array_equal(bits(f32("restored_margins.f32", (R, K))), bits(margins))
    np.testing.assert_array_equal(f32("classes.f32", (R,)), o.predict(x, objective="multi:softmax").reshape(R))
    # the probability view is the same trees under multi:softprob
    op = orc.Model(x, y.astype(np.float32), "multi:softprob", num_class=K, max_depth=4, max_bin=256, eta=0.3,
                   rounds=rounds, threads=4)
    np.testing.assert_array_equal(bits(f32("probs.f32", (R, K))), bits(op.predict(x)))
    # the slice keeps the first `cut` rounds: its trees and margins
    sliced = json.loads((tmp_path / "slice.json").read_text())["learner"]["gradient_booster"]["model"]
    assert len(sliced["trees"]) == cut * K and sliced["gbtree_model_param"]["num_trees"] == str(cut * K)
    for a, b in zip(sliced["trees"], trees[:cut * K]):
        assert a["split_conditions"] == b["split_conditions"] and a["split_indices"] == b["split_indices"]
    np.testing.assert_array_equal(bits(f32("slice_margins.f32", (R, K))),
                                  bits(o.predict(x, margin=True, iteration_end=cut)))
    session = json.loads((tmp_path / "session.json").read_text())
    assert session["train_metrics"]["CUDA_training"] is True
    assert session["slice_metrics"]["FIT_performed"] is False
    # a second trial on the same resident matrix (the search / out-of-fold reuse)
    assert session["second_metrics"]["trial"] == 2 and session["second_metrics"]["matrix_creations"] == 1
    o2 = orc.Model(x, y.astype(np.float32), "multi:softmax", num_class=K, max_depth=3, max_bin=256, eta=0.5,
                   reg_lambda=2.0, rounds=rounds, threads=4)
    trees2 = json.loads((tmp_path / "model2.json").read_text())["learner"]["gradient_booster"]["model"]["trees"]
    assert len(trees2) == o2.num_trees()
    for i, t in enumerate(trees2):
        ot = o2.tree(i)
        np.testing.assert_array_equal(np.array(t["split_indices"]), ot["split_indices"])
        np.testing.assert_array_equal(bits(t["split_conditions"]), bits(ot["split_conditions"]))
