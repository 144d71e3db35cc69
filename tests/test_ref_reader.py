"""Model JSON fidelity with the reference converter as the consumer: the
reference's own model reader (native/class_io.hpp:99-242, compiled unmodified
into oracle/_ref/ref_read_model) must accept models that libdp_gbdt writes and
read back the same thresholds, leaf values, children, default directions and
class channels, bit for bit (the fp32 round trip docs/release-validation.md:8
of the reference requires)."""
import json
import pathlib
import subprocess

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
READER = ROOT / "oracle" / "_ref" / "ref_read_model"

pytestmark = pytest.mark.skipif(not READER.exists(), reason="reference reader not built (needs the reference sources)")


def read_with_reference(path: pathlib.Path) -> dict:
    r = subprocess.run([str(READER), str(path)], capture_output=True, text=True, timeout=120)
    doc = json.loads(r.stdout)
    assert r.returncode == 0 and doc["ok"], doc
    return doc


def f32_bits(values):
    return [int(np.float32(v).view(np.uint32)) for v in values]


def check_against_trees(doc: dict, trees: list, K: int):
    """trees: dicts with left_children, right_children, split_indices,
    split_conditions (fp32), default_left, and the tree's class."""
    assert doc["outputs"] == K
    assert doc["channels"] == [t["klass"] for t in trees]
    offset = 0
    for i, t in enumerate(trees):
        n = len(t["left_children"])
        assert doc["roots"][i] == offset
        for j in range(n):
            leaf = t["left_children"][j] == -1
            g = offset + j
            assert doc["feature"][g] == (-1 if leaf else t["split_indices"][j])
            assert doc["left"][g] == (-1 if leaf else offset + t["left_children"][j])
            assert doc["right"][g] == (-1 if leaf else offset + t["right_children"][j])
            c = f32_bits([t["split_conditions"][j]])[0]
            assert (doc["value_bits"][g] if leaf else doc["cut_bits"][g]) == c
            if not leaf:
                assert doc["missing_left"][g] == int(t["default_left"][j])
        offset += n


def test_hand_written_model_survives_load_and_save(dp, tmp_path):
    """A 2-class, 2-round softprob model written here, loaded into libdp_gbdt
    and saved again, is read by the reference with every value intact
    (thresholds chosen to need all nine significant digits)."""
    def tree(i, klass, cond, leaves):
        return {"base_weights": [0.0, leaves[0], leaves[1]], "categories": [], "categories_nodes": [],
                "categories_segments": [], "categories_sizes": [], "default_left": [1, 0, 0], "id": i,
                "left_children": [1, -1, -1], "loss_changes": [1.5, 0.0, 0.0], "parents": [2147483647, 0, 0],
                "right_children": [2, -1, -1], "split_conditions": [cond, leaves[0], leaves[1]],
                "split_indices": [klass, 0, 0], "split_type": [0, 0, 0], "sum_hessian": [4.0, 2.0, 2.0],
                "tree_param": {"num_deleted": "0", "num_feature": "3", "num_nodes": "3",
                               "size_leaf_vector": "1"}}
    conds = [0.100000001, -1.23456788, 3.40282347e38, 1.17549435e-38]
    leaves = [(0.125, -0.0625), (-0.300000012, 0.300000012), (1e-30, -2.5), (0.5, 0.25)]
    trees = [tree(i, i % 2, conds[i], leaves[i]) for i in range(4)]
    model = {"learner": {
        "attributes": {}, "feature_names": [], "feature_types": [],
        "gradient_booster": {"model": {"gbtree_model_param": {"num_parallel_tree": "1", "num_trees": "4"},
                                       "iteration_indptr": [0, 2, 4], "tree_info": [0, 1, 0, 1], "trees": trees},
                             "name": "gbtree"},
        "learner_model_param": {"base_score": "[0,0]", "boost_from_average": "0", "num_class": "2",
                                "num_feature": "3", "num_target": "1"},
        "objective": {"name": "multi:softprob", "softmax_multiclass_param": {"num_class": "2"}}},
        "version": [3, 4, 1]}
    b = dp.Booster({}, [])
    b.load_raw(json.dumps(model).encode())
    saved = tmp_path / "model.json"
    saved.write_bytes(b.save_raw())
    doc = read_with_reference(saved)
    expect = [{"left_children": t["left_children"], "right_children": t["right_children"],
               "split_indices": t["split_indices"], "split_conditions": t["split_conditions"],
               "default_left": t["default_left"], "klass": i % 2} for i, t in enumerate(trees)]
    check_against_trees(doc, expect, 2)
    assert doc["features"] == 3


SHAPE = ROOT / "oracle" / "_ref" / "ref_convert_shape"


def convert_shape(path: pathlib.Path) -> dict:
    r = subprocess.run([str(SHAPE), "shape", str(path)], capture_output=True, text=True, timeout=120)
    return json.loads(r.stdout)


@pytest.mark.skipif(not SHAPE.exists(), reason="reference converter harness not built (needs the reference sources)")
@pytest.mark.parametrize("objective", ["multi:softprob", "multi:softmax", "binary:logistic"])
def test_reference_converter_source_gate(dp, tmp_path, objective):
    """The reference converter's own source gate, source_shape()
    (native/class_model_convert.cpp:49-60, compiled unmodified), on models
    saved by libdp_gbdt: gbtree, decimal num_feature / num_class /
    num_target, version 3.4.1 pass; the converter accepts only multiclass
    sources, so a binary:logistic model is refused with its own message."""
    K = 3 if objective.startswith("multi:") else 1
    trees = [{"base_weights": [0.0, 0.5, -0.5], "categories": [], "categories_nodes": [], "categories_segments": [],
              "categories_sizes": [], "default_left": [0, 0, 0], "id": i, "left_children": [1, -1, -1],
              "loss_changes": [1.0, 0.0, 0.0], "parents": [2147483647, 0, 0], "right_children": [2, -1, -1],
              "split_conditions": [0.25, 0.5, -0.5], "split_indices": [i % 4, 0, 0], "split_type": [0, 0, 0],
              "sum_hessian": [2.0, 1.0, 1.0],
              "tree_param": {"num_deleted": "0", "num_feature": "4", "num_nodes": "3", "size_leaf_vector": "1"}}
             for i in range(K)]
    obj = {"name": objective}
    if K > 1:
        obj["softmax_multiclass_param"] = {"num_class": str(K)}
    else:
        obj["reg_loss_param"] = {"scale_pos_weight": "1"}
    model = {"learner": {
        "attributes": {}, "feature_names": [], "feature_types": [],
        "gradient_booster": {"model": {"gbtree_model_param": {"num_parallel_tree": "1", "num_trees": str(K)},
                                       "iteration_indptr": [0, K], "tree_info": list(range(K)), "trees": trees},
                             "name": "gbtree"},
        "learner_model_param": {"base_score": "[" + ",".join(["0"] * K) + "]" if K > 1 else "5E-1",
                                "boost_from_average": "0", "num_class": str(K if K > 1 else 0),
                                "num_feature": "4", "num_target": "1"},
        "objective": obj},
        "version": [3, 4, 1]}
    b = dp.Booster({}, [])
    b.load_raw(json.dumps(model).encode())
    saved = tmp_path / "model.json"
    saved.write_bytes(b.save_raw())
    doc = convert_shape(saved)
    if K > 1:
        assert doc["ok"], doc
        assert (doc["features"], doc["classes"], doc["objective"]) == (4, K, objective)
    else:
        assert not doc["ok"] and doc["error"] == "source must use multiclass softprob or softmax"
