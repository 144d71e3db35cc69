"""Model JSON from a caller is checked before use.  XGBoosterLoadModel* runs
inside the caller's process on bytes the caller supplies, and a loaded
model's round index (iteration_indptr), tree classes and child ids later
index host vectors (slicing) and device arrays (prediction), so a malformed
model must be refused with -1 and a message at load, and no input may crash
the parser.  The same holds for the array interfaces that describe a caller's
matrix: a malformed one is refused before any CUDA call.  Runs on the CPU:
loading, saving and slicing touch no device."""
import copy
import ctypes as C
import json
import random

import pytest

from test_abi import _model


def load(lib, doc):
    buf = doc if isinstance(doc, bytes) else json.dumps(doc).encode()
    h = C.c_void_p()
    assert lib.XGBoosterCreate(None, 0, C.byref(h)) == 0
    rc = lib.XGBoosterLoadModelFromBuffer(h, buf, len(buf))
    msg = lib.XGBGetLastError().decode("ascii") if rc else ""  # messages are plain text
    return h, rc, msg


def edit(path, value):
    m = _model()
    node = m
    for k in path[:-1]:
        node = node[k]
    node[path[-1]] = value
    return m


MODEL = ["learner", "gradient_booster", "model"]
TREE0 = MODEL + ["trees", 0]


@pytest.mark.parametrize("doc,needle", [
    (edit(MODEL + ["iteration_indptr"], [0, 7, 2]), "iteration_indptr must be non-decreasing"),
    (edit(MODEL + ["iteration_indptr"], [0, 2, 1, 2]), "iteration_indptr must be non-decreasing"),
    (edit(MODEL + ["iteration_indptr"], [0, 3]), "iteration_indptr does not cover"),
    (edit(MODEL + ["tree_info"], [0, 2]), "tree_info names a class outside num_class"),
    (edit(MODEL + ["tree_info"], [-1, 0]), "tree_info names a class outside num_class"),
    (edit(["learner", "learner_model_param", "num_class"], "-3"), "num_class is outside"),
    (edit(["learner", "learner_model_param", "num_class"], "99999999999"), "num_class is outside"),
    (edit(TREE0 + ["left_children"], [5, -1, -1]), "tree child index out of range"),
    (edit(TREE0 + ["right_children"], [2, -1]), "tree node arrays differ in size"),
    (edit(MODEL + ["tree_info"], [0]), "tree_info size differs"),
    (edit(["learner", "learner_model_param", "base_score"], "[0.5,0.5,0.5]"), "base_score must have one value"),
    (edit(["learner", "learner_model_param", "num_feature"], "-1e+300"), "invalid integer"),
    (edit(["learner", "learner_model_param", "num_feature"], "12abc"), "invalid integer"),
    (edit(["learner", "learner_model_param", "num_feature"], "-2"), "num_feature is outside"),
])
def test_malformed_models_are_refused_at_load(dp, doc, needle):
    lib = dp.lib()
    h, rc, msg = load(lib, doc)
    lib.XGBoosterFree(h)
    assert rc == -1 and needle in msg, msg


def mutate(rng, m):
    m = copy.deepcopy(m)
    values = [-1, -2, 0, 1, 2, 3, 7, 2**31 - 1, 2**31, -2**31, 2**63 - 1, 1e300, -1e300, 0.5, "x", None, [], {},
              True, "nan", "1", "-1", "99999999999"]
    lr = m["learner"]
    model = lr["gradient_booster"]["model"]
    t = model["trees"][rng.randrange(len(model["trees"]))]
    key = rng.choice(["left_children", "right_children", "split_indices", "split_conditions", "default_left",
                      "base_weights", "sum_hessian", "loss_changes", "split_type"])
    op = rng.randrange(6)
    if op == 0 and isinstance(t.get(key), list) and t[key]:
        t[key][rng.randrange(len(t[key]))] = rng.choice(values)
    elif op == 1 and isinstance(t.get(key), list):
        t[key] = t[key][:rng.randrange(len(t[key]) + 1)]
    elif op == 2:
        t[key] = rng.choice(values)
    elif op == 3:
        t.pop(key, None)
    elif op == 4:
        model[rng.choice(["tree_info", "iteration_indptr"])] = [rng.choice(values) for _ in range(rng.randrange(5))]
    else:
        p = lr["learner_model_param"]
        p[rng.choice(sorted(p))] = str(rng.choice(values))
    return m


def test_no_input_crashes_load_save_or_slice(dp):
    lib = dp.lib()
    rng = random.Random(20240601)
    good = json.dumps(_model()).encode()
    docs = [good[:i] for i in range(0, len(good), 11)]
    for _ in range(400):
        b = bytearray(good)
        for _ in range(rng.randint(1, 4)):
            b[rng.randrange(len(b))] = rng.randrange(256)
        docs.append(bytes(b))
    docs += [b"[" * 200000 + b"]" * 200000, b'{"a":' * 50000 + b"1" + b"}" * 50000, b"1e999999", b'"\\ud800"']
    docs += [mutate(rng, mutate(rng, _model()) if rng.random() < 0.3 else _model()) for _ in range(600)]
    loaded = 0
    for doc in docs:
        h, rc, _ = load(lib, doc)
        assert rc in (0, -1)
        if rc == 0:
            loaded += 1
            n, p = C.c_uint64(), C.c_void_p()
            # what loads, saves, and what the library saves, it loads again
            assert lib.XGBoosterSaveModelToBuffer(h, b'{"format":"json"}', C.byref(n), C.byref(p)) == 0
            h2, rc2, msg2 = load(lib, C.string_at(p, n.value))
            lib.XGBoosterFree(h2)
            assert rc2 == 0, msg2
            for begin, end, step in ((0, 1, 1), (0, 0, 1), (1, 0, 1), (0, 5, 2)):
                s = C.c_void_p()
                if lib.XGBoosterSlice(h, begin, end, step, C.byref(s)) == 0:
                    lib.XGBoosterFree(s)
        lib.XGBoosterFree(h)
    assert loaded > 0  # the harmless edits still load


def raw_model(**subst):
    """The test model as JSON text with `objective` replaced by raw text."""
    text = json.dumps(_model())
    for k, v in subst.items():
        text = text.replace(k, v)
    return text.encode()


@pytest.mark.parametrize("escaped,ok", [
    (r'"\u0072eg:squarederror"', True),                       # a BMP escape of 'r'
    (r'"\ud83d\ude00"', False),                               # a surrogate pair: valid, unknown objective
    (r'"\u12G4"', False),                                      # not hex
    (r'"\ud83d"', False),                                      # lone high surrogate
    (r'"\ude00x"', False),                                     # lone low surrogate
])
def test_unicode_escapes(dp, escaped, ok):
    lib = dp.lib()
    m = _model()
    m["learner"]["objective"]["name"] = "reg:squarederror"
    m["learner"]["learner_model_param"]["num_class"] = "0"
    m["learner"]["learner_model_param"]["base_score"] = "[0]"
    m["learner"]["gradient_booster"]["model"]["tree_info"] = [0, 0]
    text = json.dumps(m).replace('"reg:squarederror"', escaped).encode()
    h, rc, msg = load(lib, text)
    lib.XGBoosterFree(h)
    if ok:
        assert rc == 0, msg
    elif "G4" in escaped or escaped.count("\\u") == 1:
        assert rc == -1 and "bad JSON unicode escape" in msg, msg
    else:
        assert rc == -1 and "objective" in msg.lower(), msg   # decoded, then refused as an objective


def test_error_messages_quote_input_as_plain_text(dp):
    lib = dp.lib()
    h, rc, msg = load(lib, b'{"version": [3, 4, 1], "learner": \xff\xfe\x01}')
    lib.XGBoosterFree(h)
    assert rc == -1 and "\\xff\\xfe\\x01" in msg, msg


def iface(**kw):
    d = {"data": [4096, True], "shape": [10, 4], "strides": None, "typestr": "<f4", "version": 3}
    d.update(kw)
    return json.dumps(d).encode()


@pytest.mark.parametrize("text,needle", [
    (iface(typestr="<f8"), "float32"),
    (iface(shape=[10, 4, 2]), "two-dimensional"),
    (iface(shape=[10, 0]), "column count out of range"),
    (iface(shape=[10, 2**31]), "column count out of range"),
    (iface(strides=[16, 8]), "row-major"),
    (iface(strides=[18, 4]), "row-major"),
    (iface(strides=[2**50, 4]), "row stride out of range"),
    (iface(shape=[2**61, 4]), "overflows"),
    (iface(data=[0, True]), "data pointer is null"),
    (iface(mask=[1]), "masked arrays"),
    (b"[" + iface() + b"," + iface() + b"]", "only one array interface"),
    (iface(data="x"), "data must be"),
    (b'{"shape": [1, 1]}', "missing JSON key"),
])
def test_malformed_array_interfaces_are_refused(dp, text, needle):
    """Checked before any CUDA call, so these run without a GPU."""
    lib = dp.lib()
    for create in (lib.XGDMatrixCreateFromCudaArrayInterface, lib.XGDMatrixCreateFromDense):
        h = C.c_void_p()
        assert create(text, b'{"missing": NaN}', C.byref(h)) == -1
        msg = lib.XGBGetLastError().decode("ascii")
        assert needle in msg, msg


@pytest.mark.parametrize("config,needle", [
    ({"type": 2}, "type is out of range"),
    ({"type": 2**32}, "type is out of range"),
    ({"iteration_begin": -1}, "iteration_begin is out of range"),
    ({"iteration_end": 2**32 + 1}, "iteration_end is out of range"),
    ({"iteration_end": 5}, "iteration range outside the model's rounds"),
])
def test_prediction_config_is_checked_before_device_work(dp, config, needle):
    """A value that would wrap when narrowed (2^32 + 1 -> 1) is refused, not
    read as another, valid-looking one."""
    lib = dp.lib()
    h, rc, _ = load(lib, _model())
    assert rc == 0
    shape, dims, out = C.POINTER(C.c_uint64)(), C.c_uint64(), C.POINTER(C.c_float)()
    cfg = json.dumps(dict({"missing": float("nan")}, **config)).encode()
    rc = lib.XGBoosterPredictFromCudaArray(h, iface(shape=[10, 2]), cfg, None, C.byref(shape), C.byref(dims),
                                           C.byref(out))
    msg = lib.XGBGetLastError().decode("ascii")
    lib.XGBoosterFree(h)
    assert rc == -1 and needle in msg, msg


@pytest.mark.parametrize("shape,strides,needle", [
    ([10, 1], [16, 4], "contiguous"),       # a column of a 4-wide matrix
    ([10], [8], "contiguous"),
    ([10], [4, 4], "contiguous"),
    ([10, 2], None, "vector"),
    ([10, 1, 1], None, "vector"),
])
def test_label_interfaces_are_checked_before_the_matrix(dp, shape, strides, needle):
    """Label arrays are checked before the matrix handle is used (here a null
    one), so these run without a GPU."""
    lib = dp.lib()
    rc = lib.XGDMatrixSetInfoFromInterface(None, b"label", iface(shape=shape, strides=strides))
    msg = lib.XGBGetLastError().decode("ascii")
    assert rc == -1 and needle in msg, msg


def test_contiguous_label_interfaces_reach_the_matrix_check(dp):
    lib = dp.lib()
    for shape, strides in (([10], None), ([10], [4]), ([10, 1], [4, 4]), ([1, 1], [64, 4])):
        rc = lib.XGDMatrixSetInfoFromInterface(None, b"label", iface(shape=shape, strides=strides))
        msg = lib.XGBGetLastError().decode("ascii")
        assert rc == -1 and "DMatrix handle is null" in msg, (shape, strides, msg)


def test_null_output_pointers_are_refused(dp):
    """Where XGBoost returns an error for a null output pointer, so does this
    library, instead of writing through it."""
    lib = dp.lib()
    h, rc, _ = load(lib, _model())
    assert rc == 0
    n, p = C.c_uint64(), C.c_void_p()
    calls = [
        lambda: lib.XGBoosterGetNumFeature(h, None),
        lambda: lib.XGBoosterSaveJsonConfig(h, None, None),
        lambda: lib.XGBoosterSaveJsonConfig(h, C.byref(n), None),
        lambda: lib.XGBoosterSaveModelToBuffer(h, b'{"format":"json"}', None, None),
        lambda: lib.XGBoosterSaveModelToBuffer(h, b'{"format":"json"}', C.byref(n), None),
        lambda: lib.dp_booster_profile(h, None),
    ]
    for i, call in enumerate(calls):
        assert call() == -1, i
        assert "null" in lib.XGBGetLastError().decode("ascii"), i
    assert lib.XGBoosterSaveModelToBuffer(h, b'{"format":"json"}', C.byref(n), C.byref(p)) == 0 and n.value > 0
    lib.XGBoosterFree(h)


def test_parameters_never_crash_or_break_the_configuration(dp):
    """Random keys and values through XGBoosterSetParam: every call returns 0
    or -1 with a plain-text message, and the configuration document stays
    valid JSON whatever was recorded (quotes, backslashes, control bytes)."""
    lib = dp.lib()
    rng = random.Random(7)
    keys = ["objective", "num_class", "max_depth", "max_bin", "eta", "lambda", "alpha", "gamma", "min_child_weight",
            "subsample", "colsample_bynode", "seed", "device", "tree_method", "base_score", "max_delta_step",
            "num_parallel_tree", "nthread", "eval_metric", "", "k\"ey", "\xff"]
    values = ["", "0", "1", "-1", "1e309", "nan", "inf", "0.5", "2", "256", "99999999999999999999", "cuda:", "cuda:0",
              "cuda:-1", "cuda:99999999999", "cpu", "\"quoted\"", "\"", "[0.5]", "[", "hist", "multi:softprob",
              "a\\b", "\x01", "\xff\xfe", "0x10", "1e-400", "{}"]
    for _ in range(1500):
        h = C.c_void_p()
        assert lib.XGBoosterCreate(None, 0, C.byref(h)) == 0
        for _ in range(rng.randint(1, 4)):
            rc = lib.XGBoosterSetParam(h, rng.choice(keys).encode("latin-1"), rng.choice(values).encode("latin-1"))
            assert rc in (0, -1)
            if rc:
                lib.XGBGetLastError().decode("ascii")
        n, s = C.c_uint64(), C.c_char_p()
        assert lib.XGBoosterSaveJsonConfig(h, C.byref(n), C.byref(s)) == 0
        json.loads(C.string_at(s, n.value))
        lib.XGBoosterFree(h)


def test_boundary_calls_from_many_threads(dp):
    """Searches and out-of-fold fits may drive boosters from several threads:
    load, save, slice and refusals run concurrently, every thread reads its
    own error message, and every saved model is the same text."""
    import threading
    lib = dp.lib()
    good = json.dumps(_model()).encode()
    bad = good[:-5]
    outs, errors = [], []

    def work(tid):
        try:
            for i in range(120):
                h = C.c_void_p()
                assert lib.XGBoosterCreate(None, 0, C.byref(h)) == 0
                if (i + tid) % 3 == 0:
                    assert lib.XGBoosterLoadModelFromBuffer(h, bad, len(bad)) == -1
                    assert "JSON" in lib.XGBGetLastError().decode("ascii")
                assert lib.XGBoosterLoadModelFromBuffer(h, good, len(good)) == 0
                n, p = C.c_uint64(), C.c_void_p()
                assert lib.XGBoosterSaveModelToBuffer(h, b'{"format":"json"}', C.byref(n), C.byref(p)) == 0
                outs.append(C.string_at(p, n.value))
                s = C.c_void_p()
                assert lib.XGBoosterSlice(h, 0, 1, 1, C.byref(s)) == 0
                lib.XGBoosterFree(s)
                lib.XGBoosterFree(h)
        except Exception as e:  # reported below, from the main thread
            errors.append(repr(e))

    threads = [threading.Thread(target=work, args=(t,)) for t in range(8)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors[:3]
    assert len(outs) == 8 * 120 and len(set(outs)) == 1


@pytest.mark.parametrize("source", ["param", "model"])
def test_prediction_without_classes_is_refused_on_the_host(dp, source):
    """multi:softprob with num_class 0 (a parameter, or a tree-less model
    file) has outputs [rows][0]; predicting is refused before device work
    instead of transforming an empty margin buffer."""
    lib = dp.lib()
    if source == "param":
        h = C.c_void_p()
        assert lib.XGBoosterCreate(None, 0, C.byref(h)) == 0
        assert lib.XGBoosterSetParam(h, b"objective", b"multi:softprob") == 0
        assert lib.XGBoosterSetParam(h, b"num_class", b"0") == 0
    else:
        m = _model()
        m["learner"]["learner_model_param"]["num_class"] = "0"
        m["learner"]["learner_model_param"]["base_score"] = "[0]"
        model = m["learner"]["gradient_booster"]["model"]
        model["trees"], model["tree_info"], model["iteration_indptr"] = [], [], [0]
        h, rc, msg = load(lib, m)
        assert rc == 0, msg
    shape, dims, out = C.POINTER(C.c_uint64)(), C.c_uint64(), C.POINTER(C.c_float)()
    rc = lib.XGBoosterPredictFromCudaArray(h, iface(shape=[10, 2]), b'{"type": 0, "missing": NaN}', None,
                                           C.byref(shape), C.byref(dims), C.byref(out))
    msg = lib.XGBGetLastError().decode("ascii")
    lib.XGBoosterFree(h)
    assert rc == -1 and "num_class must be at least 1" in msg, msg


def test_kernel_level_entry_points_refuse_null_pointers(dp):
    """The kernel-level entry points take device pointers; a missing one is
    refused on the host before any device work, instead of a kernel writing
    through it."""
    lib = dp.lib()
    seg_b = (C.c_int64 * 1)(0)
    seg_e = (C.c_int64 * 1)(10)
    fake = 4096  # never dereferenced: every call below is refused first
    out_i, gain, left = (C.c_int32 * 4)(), (C.c_double * 1)(), (C.c_int64 * 2)()
    totals = (C.c_int64 * 2)(1, 1)
    calls = {
        "quantile cuts output": lambda: lib.dp_quantile_cuts(fake, 10, 2, 2, 256, None, fake, fake, None),
        "quantile cuts input": lambda: lib.dp_quantile_cuts(None, 10, 2, 2, 256, fake, fake, fake, None),
        "quantile cuts stride": lambda: lib.dp_quantile_cuts(fake, 10, 4, 2, 256, fake, fake, fake, None),
        "bin matrix bins": lambda: lib.dp_bin_matrix(fake, 10, 2, 2, fake, fake, None, 16, None),
        "bin matrix cuts": lambda: lib.dp_bin_matrix(fake, 10, 2, 2, None, fake, fake, 16, None),
        "gradients": lambda: lib.dp_gradients(0, 1, None, fake, 10, fake, fake, None),
        "gradient scales": lambda: lib.dp_gradients(0, 1, fake, fake, 10, fake, None, None),
        "quantize": lambda: lib.dp_quantize_gh(None, 10, 1.0, 1.0, None),
        "eval input": lambda: lib.dp_eval_splits(None, 1, 2, fake, fake, totals, 1.0, 1.0, 1.0, 0.0, 0.0, 1.0,
                                                 out_i, gain, left),
        "eval output": lambda: lib.dp_eval_splits(fake, 1, 2, fake, fake, totals, 1.0, 1.0, 1.0, 0.0, 0.0, 1.0,
                                                  None, gain, left),
        "no-allocation hist": lambda: lib.dp_hist_build_noalloc(fake, 16, 2, 256, fake, fake, seg_b, seg_e, 1,
                                                                1.0, 1.0, None, None),
        "no-allocation bins": lambda: lib.dp_hist_build_noalloc(None, 16, 2, 256, fake, fake, seg_b, seg_e, 1,
                                                                1.0, 1.0, fake, None),
    }
    for name, call in calls.items():
        assert call() == -1, name
        msg = lib.XGBGetLastError().decode("ascii")
        assert "null" in msg or "cover the features" in msg, (name, msg)


def test_base_score_of_the_wrong_length_is_named(dp):
    """base_score set as a vector must have one value per class; a mismatch
    is reported as such when the model is saved (or trained or used)."""
    lib = dp.lib()
    h = C.c_void_p()
    assert lib.XGBoosterCreate(None, 0, C.byref(h)) == 0
    assert lib.XGBoosterSetParam(h, b"objective", b"reg:squarederror") == 0
    assert lib.XGBoosterSetParam(h, b"base_score", b"[0.5, 0.2]") == 0
    n, p = C.c_uint64(), C.c_void_p()
    rc = lib.XGBoosterSaveModelToBuffer(h, b'{"format":"json"}', C.byref(n), C.byref(p))
    msg = lib.XGBGetLastError().decode("ascii")
    assert rc == -1 and "base_score must have one value or one per class" in msg, msg
    assert lib.XGBoosterSetParam(h, b"base_score", b"[0.5]") == 0
    assert lib.XGBoosterSaveModelToBuffer(h, b'{"format":"json"}', C.byref(n), C.byref(p)) == 0
    lib.XGBoosterFree(h)


def test_saved_models_reload_to_the_same_text(dp):
    """For random objective, class and base_score settings: a model that
    saves loads again, and saving it again gives the same text."""
    lib = dp.lib()
    rng = random.Random(5)
    keys = ["objective", "num_class", "base_score", "max_depth", "eta", "seed"]
    values = ["reg:squarederror", "binary:logistic", "multi:softprob", "multi:softmax", "0", "1", "2", "3", "0.5",
              "[0.5]", "[0.2,0.3]", "[0.1,0.2,0.3]", "[]", "-1", "nan"]
    saved = 0
    for _ in range(2000):
        h = C.c_void_p()
        assert lib.XGBoosterCreate(None, 0, C.byref(h)) == 0
        for _ in range(rng.randint(1, 6)):
            lib.XGBoosterSetParam(h, rng.choice(keys).encode(), rng.choice(values).encode())
        n, p = C.c_uint64(), C.c_void_p()
        if lib.XGBoosterSaveModelToBuffer(h, b'{"format":"json"}', C.byref(n), C.byref(p)) == 0:
            text = C.string_at(p, n.value)
            h2, rc, msg = load(lib, text)
            assert rc == 0, msg
            assert lib.XGBoosterSaveModelToBuffer(h2, b'{"format":"json"}', C.byref(n), C.byref(p)) == 0
            assert C.string_at(p, n.value) == text
            lib.XGBoosterFree(h2)
            saved += 1
        lib.XGBoosterFree(h)
    assert saved > 1000
