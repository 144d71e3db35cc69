"""ctypes binding of libdp_gbdt (include/dp_gbdt.h).

Mirrors the call sequence the reference trainer issues through the XGBoost C
API (native/class_native_training.cuh:47-70): a DMatrix over borrowed CUDA
fp32 memory, a Booster configured with XGBoosterSetParam, one
XGBoosterUpdateOneIter per round, then the JSON configuration and model.
Device memory is supplied by the caller (here: torch CUDA tensors or raw
pointers); the library itself has no CPU training path and raises if its
shared object is missing.
"""
from __future__ import annotations

import ctypes as C
import json
import math
import pathlib
from typing import Iterable

HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = HERE / "libdp_gbdt.so"

EXPORTED = [
    "XGBoostVersion", "XGBuildInfo", "XGBGetLastError", "XGDMatrixCreateFromCudaArrayInterface",
    "XGDMatrixCreateFromDense",
    "XGDMatrixSetInfoFromInterface", "XGDMatrixSetFloatInfo", "XGDMatrixNumRow", "XGDMatrixNumCol",
    "XGDMatrixFree", "XGBoosterCreate", "XGBoosterFree", "XGBoosterSetParam", "XGBoosterUpdateOneIter",
    "XGBoosterBoostedRounds", "XGBoosterSaveJsonConfig", "XGBoosterSaveModel", "XGBoosterSaveModelToBuffer",
    "XGBoosterLoadModelFromBuffer", "XGBoosterLoadModel", "XGBoosterSlice", "XGBoosterGetNumFeature",
    "XGBoosterPredictFromCudaArray",
    "dp_comm_unique_id", "dp_comm_create", "dp_comm_free", "dp_comm_set_timeout", "dp_comm_reduce_scatter_hist", "dp_release_cached_memory", "dp_booster_set_comm", "dp_booster_set_profiling",
    "dp_booster_profile", "dp_booster_margins", "dp_launch_count", "dp_quantile_cuts", "dp_bin_matrix",
    "dp_gradients", "dp_hist_build", "dp_hist_build_noalloc", "dp_probe_hist_atomics", "dp_csv_decode", "dp_csv_shape", "dp_csv_data", "dp_csv_metadata", "dp_csv_copy", "dp_csv_free", "dp_csv_parse_feature", "dp_quantize_gh", "dp_hist_prepare", "dp_hist_run", "dp_hist_free", "dp_eval_splits",
]

OBJECTIVE_IDS = {"reg:squarederror": 0, "binary:logistic": 1, "multi:softprob": 2, "multi:softmax": 3}


class DPError(RuntimeError):
    pass


_lib = None


def lib() -> C.CDLL:
    """Loads libdp_gbdt.so (built by `make -C decision-programs_b200`)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise DPError(f"libdp_gbdt.so is missing at {LIB_PATH}; build it with __graft_entry__.build()")
        L = C.CDLL(str(LIB_PATH))
        P, u64, i32, f32, f64 = C.c_void_p, C.c_uint64, C.c_int, C.c_float, C.c_double
        L.XGBoostVersion.restype = None
        L.XGBoostVersion.argtypes = [C.POINTER(i32)] * 3
        L.XGBuildInfo.argtypes = [C.POINTER(C.c_char_p)]
        L.XGBGetLastError.restype = C.c_char_p
        L.XGDMatrixCreateFromCudaArrayInterface.argtypes = [C.c_char_p, C.c_char_p, C.POINTER(P)]
        L.XGDMatrixCreateFromDense.argtypes = [C.c_char_p, C.c_char_p, C.POINTER(P)]
        L.XGDMatrixSetInfoFromInterface.argtypes = [P, C.c_char_p, C.c_char_p]
        L.XGDMatrixSetFloatInfo.argtypes = [P, C.c_char_p, P, u64]
        L.XGDMatrixNumRow.argtypes = [P, C.POINTER(u64)]
        L.XGDMatrixNumCol.argtypes = [P, C.POINTER(u64)]
        L.XGDMatrixFree.argtypes = [P]
        L.XGBoosterCreate.argtypes = [C.POINTER(P), u64, C.POINTER(P)]
        L.XGBoosterFree.argtypes = [P]
        L.XGBoosterSetParam.argtypes = [P, C.c_char_p, C.c_char_p]
        L.XGBoosterUpdateOneIter.argtypes = [P, i32, P]
        L.XGBoosterBoostedRounds.argtypes = [P, C.POINTER(i32)]
        L.XGBoosterSaveJsonConfig.argtypes = [P, C.POINTER(u64), C.POINTER(C.c_char_p)]
        L.XGBoosterSaveModel.argtypes = [P, C.c_char_p]
        L.XGBoosterSaveModelToBuffer.argtypes = [P, C.c_char_p, C.POINTER(u64), C.POINTER(C.c_void_p)]
        L.XGBoosterLoadModelFromBuffer.argtypes = [P, C.c_char_p, u64]
        L.XGBoosterLoadModel.argtypes = [P, C.c_char_p]
        L.XGBoosterSlice.argtypes = [P, i32, i32, i32, C.POINTER(P)]
        L.XGBoosterGetNumFeature.argtypes = [P, C.POINTER(u64)]
        L.XGBoosterPredictFromCudaArray.argtypes = [P, C.c_char_p, C.c_char_p, P, C.POINTER(C.POINTER(u64)),
                                                    C.POINTER(u64), C.POINTER(C.POINTER(f32))]
        L.dp_comm_unique_id.argtypes = [P]
        L.dp_comm_create.argtypes = [P, i32, i32, i32, C.POINTER(P)]
        L.dp_comm_free.argtypes = [P]
        L.dp_comm_set_timeout.argtypes = [P, C.c_int64]
        L.dp_comm_reduce_scatter_hist.argtypes = [P, P, P, u64, P]
        L.dp_release_cached_memory.argtypes = []
        L.dp_booster_set_comm.argtypes = [P, P]
        L.dp_booster_set_profiling.argtypes = [P, i32]
        L.dp_booster_profile.argtypes = [P, C.POINTER(C.c_char_p)]
        L.dp_booster_margins.argtypes = [P, P, u64]
        L.dp_launch_count.restype = u64
        L.dp_launch_count.argtypes = []
        L.dp_quantile_cuts.argtypes = [P, u64, C.c_uint32, u64, i32, P, P, P, P]
        L.dp_bin_matrix.argtypes = [P, u64, C.c_uint32, u64, P, P, P, u64, P]
        L.dp_gradients.argtypes = [i32, i32, P, P, u64, P, P, P]
        L.dp_hist_build.argtypes = [P, u64, C.c_uint32, C.c_int32, P, P, P, P, C.c_int32, f32, f32, P, P]
        L.dp_hist_build_noalloc.argtypes = [P, u64, C.c_uint32, C.c_int32, P, P, P, P, C.c_int32, f32, f32, P, P]
        L.dp_quantize_gh.argtypes = [P, u64, f32, f32, P]
        L.dp_probe_hist_atomics.argtypes = [C.c_uint32, C.POINTER(C.c_double), P]
        L.dp_csv_decode.argtypes = [C.c_char_p, u64, C.c_char_p, C.c_char_p, P, C.POINTER(P)]
        L.dp_csv_shape.argtypes = [P, C.POINTER(u64), C.POINTER(C.c_uint32), C.POINTER(C.c_uint32),
                                   C.POINTER(C.c_int32)]
        L.dp_csv_data.argtypes = [P, C.POINTER(P), C.POINTER(P)]
        L.dp_csv_metadata.argtypes = [P, C.POINTER(C.c_char_p), C.POINTER(C.c_double)]
        L.dp_csv_copy.argtypes = [P, P, P]
        L.dp_csv_free.argtypes = [P]
        L.dp_csv_parse_feature.argtypes = [C.c_char_p, u64, C.POINTER(C.c_float)]
        L.dp_hist_prepare.argtypes = [P, u64, C.c_uint32, C.c_int32, C.c_int32, P, P, P, P, C.c_int32, f32, f32,
                                      P, C.POINTER(P)]
        L.dp_hist_run.argtypes = [P, P]
        L.dp_hist_free.argtypes = [P]
        L.dp_eval_splits.argtypes = [P, C.c_int32, C.c_uint32, P, P, P, f32, f32, f64, f64, f64, f64, P, P, P]
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != 0:
        raise DPError(lib().XGBGetLastError().decode())


def version() -> tuple[int, int, int]:
    a, b, c = C.c_int(), C.c_int(), C.c_int()
    lib().XGBoostVersion(C.byref(a), C.byref(b), C.byref(c))
    return a.value, b.value, c.value


def build_info() -> dict:
    p = C.c_char_p()
    check(lib().XGBuildInfo(C.byref(p)))
    return json.loads(p.value.decode())


def launch_count() -> int:
    return int(lib().dp_launch_count())


def array_interface(ptr: int, shape: Iterable[int], typestr: str = "<f4", strides=None) -> str:
    """__cuda_array_interface__ JSON as the reference builds it
    (native/class_model_native_adapter.cuh:26)."""
    return json.dumps({"data": [int(ptr), True], "shape": list(shape), "strides": strides, "typestr": typestr,
                       "version": 3, "stream": 1}, separators=(",", ":"))


class DMatrix:
    """Dense fp32 matrix [R][F] (NaN = missing): a borrowed CUDA matrix, or a
    host matrix copied to the current CUDA device (from_host)."""

    def __init__(self, data_ptr: int, rows: int, cols: int, label_ptr: int | None = None, row_stride: int | None = None,
                 missing: float = math.nan, keepalive=None):
        self.handle = C.c_void_p()
        strides = None if row_stride is None else [int(row_stride) * 4, 4]
        cfg = '{"missing":NaN,"nthread":2}' if math.isnan(missing) else json.dumps({"missing": missing, "nthread": 2})
        check(lib().XGDMatrixCreateFromCudaArrayInterface(array_interface(data_ptr, [rows, cols], strides=strides)
                                                          .encode(), cfg.encode(), C.byref(self.handle)))
        self._keep = keepalive
        if label_ptr is not None:
            self.set_label_ptr(label_ptr, rows)

    @classmethod
    def from_torch(cls, x, y=None, missing: float = math.nan) -> "DMatrix":
        """x: CUDA float32 tensor [R, F] (row stride allowed); y: CUDA float32 [R]."""
        assert x.is_cuda and x.dtype.is_floating_point and x.element_size() == 4 and x.dim() == 2
        assert x.stride(1) == 1
        d = cls(x.data_ptr(), x.shape[0], x.shape[1], row_stride=x.stride(0) if x.stride(0) != x.shape[1] else None,
                missing=missing, keepalive=(x, y))
        if y is not None:
            y = y.contiguous()
            d._keep = (x, y)
            d.set_label_ptr(y.data_ptr(), y.shape[0])
        return d

    @classmethod
    def from_host(cls, x, y=None, missing: float = math.nan) -> "DMatrix":
        """x: host float32 [R, F] (numpy array or CPU torch tensor, rows
        contiguous; pinned memory copies fastest); y: host float32 [R].
        Goes through XGDMatrixCreateFromDense."""
        if hasattr(x, "data_ptr"):
            assert not x.is_cuda and x.dim() == 2 and x.element_size() == 4 and x.stride(1) == 1
            ptr, (rows, cols), row_stride = x.data_ptr(), x.shape, x.stride(0)
        else:
            import numpy as np
            assert x.dtype == np.float32 and x.ndim == 2 and x.strides[1] == 4
            ptr, (rows, cols), row_stride = x.ctypes.data, x.shape, x.strides[0] // 4
        d = cls.__new__(cls)
        d.handle = C.c_void_p()
        strides = None if row_stride == cols else [int(row_stride) * 4, 4]
        cfg = '{"missing":NaN,"nthread":2}' if math.isnan(missing) else json.dumps({"missing": missing, "nthread": 2})
        check(lib().XGDMatrixCreateFromDense(array_interface(ptr, [rows, cols], strides=strides).encode(),
                                             cfg.encode(), C.byref(d.handle)))
        d._keep = None  # the library holds its own copy
        if y is not None:
            d.set_label_host(y.numpy() if hasattr(y, "numpy") else y)
        return d

    def set_label_ptr(self, ptr: int, n: int) -> None:
        check(lib().XGDMatrixSetInfoFromInterface(self.handle, b"label", array_interface(ptr, [n]).encode()))

    def set_label_host(self, y) -> None:
        import numpy as np
        y = np.ascontiguousarray(y, dtype=np.float32)
        check(lib().XGDMatrixSetFloatInfo(self.handle, b"label", y.ctypes.data, y.size))

    def num_row(self) -> int:
        n = C.c_uint64()
        check(lib().XGDMatrixNumRow(self.handle, C.byref(n)))
        return n.value

    def num_col(self) -> int:
        n = C.c_uint64()
        check(lib().XGDMatrixNumCol(self.handle, C.byref(n)))
        return n.value

    def free(self) -> None:
        if self.handle:
            check(lib().XGDMatrixFree(self.handle))
            self.handle = C.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Booster:
    def __init__(self, params: dict | None = None, cache: list[DMatrix] | None = None, handle=None):
        if handle is not None:
            self.handle = handle
        else:
            self.handle = C.c_void_p()
            cache = cache or []
            arr = (C.c_void_p * max(1, len(cache)))(*[d.handle for d in cache])
            check(lib().XGBoosterCreate(arr, len(cache), C.byref(self.handle)))
        for k, v in (params or {}).items():
            self.set_param(k, v)

    def set_param(self, key: str, value) -> None:
        if isinstance(value, (list, tuple)):
            value = json.dumps(list(value))
        elif isinstance(value, bool):
            value = "1" if value else "0"
        check(lib().XGBoosterSetParam(self.handle, key.encode(), str(value).encode()))

    def update(self, dtrain: DMatrix, iteration: int) -> None:
        check(lib().XGBoosterUpdateOneIter(self.handle, iteration, dtrain.handle))

    def boosted_rounds(self) -> int:
        n = C.c_int()
        check(lib().XGBoosterBoostedRounds(self.handle, C.byref(n)))
        return n.value

    def save_config(self) -> dict:
        n = C.c_uint64()
        p = C.c_char_p()
        check(lib().XGBoosterSaveJsonConfig(self.handle, C.byref(n), C.byref(p)))
        return json.loads(C.string_at(p, n.value).decode())

    def save_raw(self) -> bytes:
        n = C.c_uint64()
        p = C.c_void_p()
        check(lib().XGBoosterSaveModelToBuffer(self.handle, b'{"format":"json"}', C.byref(n), C.byref(p)))
        return C.string_at(p, n.value)

    def save_model(self, path: str) -> None:
        check(lib().XGBoosterSaveModel(self.handle, str(path).encode()))

    def load_raw(self, raw: bytes) -> None:
        check(lib().XGBoosterLoadModelFromBuffer(self.handle, raw, len(raw)))

    def load_model(self, path: str) -> None:
        check(lib().XGBoosterLoadModel(self.handle, str(path).encode()))

    def slice(self, begin: int, end: int, step: int = 1) -> "Booster":
        out = C.c_void_p()
        check(lib().XGBoosterSlice(self.handle, begin, end, step, C.byref(out)))
        return Booster(handle=out)

    def num_features(self) -> int:
        n = C.c_uint64()
        check(lib().XGBoosterGetNumFeature(self.handle, C.byref(n)))
        return n.value

    def set_comm(self, comm: "Comm") -> None:
        check(lib().dp_booster_set_comm(self.handle, comm.handle))

    def set_profiling(self, on, histograms_only: bool = False) -> None:
        """Mode 1 (on=True): every instrumented launch; histograms_only: mode 2;
        on=False: off.  Enabling resets the counters."""
        mode = 0 if not on else (2 if histograms_only else 1)
        check(lib().dp_booster_set_profiling(self.handle, mode))

    def profile(self) -> dict:
        p = C.c_char_p()
        check(lib().dp_booster_profile(self.handle, C.byref(p)))
        return json.loads(p.value.decode())

    def predict(self, x, margin: bool = False, iteration_begin: int = 0, iteration_end: int = 0,
                strict_shape: bool = True, missing: float = math.nan):
        """XGBoosterPredictFromCudaArray over a CUDA float32 tensor [R, F]
        (row stride allowed).  Returns a new CUDA tensor holding a copy of the
        booster-owned output, shaped as the call reports it."""
        import torch
        assert x.is_cuda and x.dtype == torch.float32 and x.dim() == 2 and x.stride(1) == 1
        strides = None if x.stride(0) == x.shape[1] else [int(x.stride(0)) * 4, 4]
        cfg = {"type": 1 if margin else 0, "training": False, "iteration_begin": iteration_begin,
               "iteration_end": iteration_end, "strict_shape": strict_shape, "cache_id": 0}
        text = json.dumps(cfg, separators=(",", ":"))[:-1] + (',"missing":NaN}' if math.isnan(missing)
                                                               else f',"missing":{missing!r}}}')
        shape = C.POINTER(C.c_uint64)()
        dims = C.c_uint64()
        out = C.POINTER(C.c_float)()
        check(lib().XGBoosterPredictFromCudaArray(self.handle, array_interface(x.data_ptr(), list(x.shape),
                                                                               strides=strides).encode(),
                                                  text.encode(), None, C.byref(shape), C.byref(dims),
                                                  C.byref(out)))
        dims_t = tuple(shape[i] for i in range(dims.value))
        n = 1
        for d in dims_t:
            n *= d
        res = torch.empty(dims_t, dtype=torch.float32, device=x.device)
        if n:
            from cuda.bindings import runtime as rt
            err, = rt.cudaMemcpy(res.data_ptr(), C.cast(out, C.c_void_p).value, n * 4,
                                 rt.cudaMemcpyKind.cudaMemcpyDeviceToDevice)
            if err != rt.cudaError_t.cudaSuccess:
                raise DPError(f"copy of the prediction failed: {err}")
        return res

    def margins(self, rows: int, outputs: int):
        import numpy as np
        out = np.zeros((rows, outputs), np.float32)
        check(lib().dp_booster_margins(self.handle, out.ctypes.data, out.size))
        return out

    def trees(self) -> list[dict]:
        return json.loads(self.save_raw())["learner"]["gradient_booster"]["model"]["trees"]

    def free(self) -> None:
        if self.handle:
            check(lib().XGBoosterFree(self.handle))
            self.handle = C.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Comm:
    """NCCL communicator for row-sharded training (one process per GPU)."""

    @staticmethod
    def unique_id() -> bytes:
        buf = C.create_string_buffer(128)
        check(lib().dp_comm_unique_id(buf))
        return buf.raw

    def __init__(self, unique_id: bytes, nranks: int, rank: int, device: int):
        assert len(unique_id) == 128
        self.handle = C.c_void_p()
        check(lib().dp_comm_create(unique_id, nranks, rank, device, C.byref(self.handle)))

    def set_timeout(self, ms: int) -> None:
        """Deadline of every host wait on collectives in flight; a peer that
        stops or fails aborts the communicator and the training call raises."""
        check(lib().dp_comm_set_timeout(self.handle, int(ms)))

    def reduce_scatter_hist(self, send_ptr: int, recv_ptr: int, recv_n: int, stream: int | None = None) -> None:
        """The sharded path's histogram exchange (int64 partial sums)."""
        check(lib().dp_comm_reduce_scatter_hist(self.handle, send_ptr, recv_ptr, recv_n, stream))

    def free(self) -> None:
        if self.handle:
            check(lib().dp_comm_free(self.handle))
            self.handle = C.c_void_p()


class CsvTable:
    """The GPU CSV decoder (dp_csv_decode): the reference's
    decision_programs_csv::decode (native/decision_programs_csv.hpp:36-67).
    `values_ptr` / `labels_ptr` are device pointers owned by this object."""

    def __init__(self, data: bytes, target: str | None = None, header: str = "auto"):
        h = C.c_void_p()
        check(lib().dp_csv_decode(data, len(data), (target or "").encode(), header.encode(), None, C.byref(h)))
        self.handle = h
        rows, feats, classes, hdr = C.c_uint64(), C.c_uint32(), C.c_uint32(), C.c_int32()
        check(lib().dp_csv_shape(h, C.byref(rows), C.byref(feats), C.byref(classes), C.byref(hdr)))
        self.rows, self.features, self.classes, self.header = rows.value, feats.value, classes.value, bool(hdr.value)
        meta, ms = C.c_char_p(), C.c_double()
        check(lib().dp_csv_metadata(h, C.byref(meta), C.byref(ms)))
        m = json.loads(meta.value.decode())
        self.names, self.label_mapping, self.device_ms = m["names"], m["label_mapping"], ms.value
        v, lb = C.c_void_p(), C.c_void_p()
        check(lib().dp_csv_data(h, C.byref(v), C.byref(lb)))
        self.values_ptr, self.labels_ptr = v.value, lb.value

    def to_numpy(self):
        import numpy as np
        values = np.empty((self.rows, self.features), np.float32)
        labels = np.empty(self.rows, np.uint32) if self.labels_ptr else None
        check(lib().dp_csv_copy(self.handle, values.ctypes.data,
                                labels.ctypes.data if labels is not None else None))
        return values, labels

    def free(self) -> None:
        if self.handle:
            check(lib().dp_csv_free(self.handle))
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def train(params: dict, dtrain: DMatrix, rounds: int, comm: Comm | None = None) -> Booster:
    """The reference's sequence: create, set params, one UpdateOneIter per round."""
    b = Booster(params, [dtrain])
    if comm is not None:
        b.set_comm(comm)
    for i in range(rounds):
        b.update(dtrain, i)
    return b
