"""TEST INFRASTRUCTURE ONLY: ctypes wrapper of the CPU oracle (liboracle.so).

The oracle restates the GBDT training arithmetic that the reference trainer
reaches through XGBoost 3.4.1 (native/class_native_training.cuh:47-70).
Parity is unpinned (no reference test pins training numerics); see the header
of gbdt_oracle.cpp for the exact semantics.  Only tests/, the smoke check and
bench.py's CPU leg import this module.
"""
from __future__ import annotations

import ctypes as C
import os
import pathlib

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

OBJECTIVES = {"reg:squarederror": 0, "binary:logistic": 1, "multi:softprob": 2, "multi:softmax": 3}

_lib = None

# all-reduce callback of the sharded runs: (int64* buf, n, op 0=sum 1=max, ctx)
ALLREDUCE = C.CFUNCTYPE(None, C.POINTER(C.c_int64), C.c_int64, C.c_int, C.c_void_p)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"oracle library missing: {LIB_PATH} (run make -C oracle)")
        L = C.CDLL(str(LIB_PATH))
        P = C.c_void_p
        u64, u32, i32, i64 = C.c_uint64, C.c_uint32, C.c_int, C.c_int64
        L.orc_exp.restype = C.c_double
        L.orc_exp.argtypes = [C.c_double]
        L.orc_cuts.argtypes = [P, u64, u32, u64, i32, i32, C.c_float, P, P, P, i32]
        L.orc_bin_matrix.argtypes = [P, u64, u32, u64, P, P, P, i32, C.c_float, P, u64, i32]
        L.orc_gradients.argtypes = [i32, i32, P, P, u64, P, i32]
        L.orc_quantizer.argtypes = [P, u64, P, P]
        L.orc_histograms.argtypes = [P, u64, u32, P, P, P, P, i64, C.c_float, C.c_float, P, i32]
        L.orc_best_splits.argtypes = [P, i64, u32, P, P, P, C.c_float, C.c_float, C.c_double, C.c_double,
                                      C.c_double, C.c_double, P, P, P]
        L.orc_train.restype = P
        L.orc_train.argtypes = [P, u64, u32, u64, P, i32, i32, i32, i32, C.c_double, C.c_double, C.c_double,
                                C.c_double, C.c_double, C.c_float, i32, i32, i32]
        L.orc_train_sharded.restype = P
        L.orc_train_sharded.argtypes = [P, u64, u32, u64, P, i32, i32, i32, i32, C.c_double, C.c_double, C.c_double,
                                        C.c_double, C.c_double, C.c_float, i32, i32, ALLREDUCE, P]
        L.orc_radix_cuts.argtypes = [P, u64, u32, u64, i32, i32, C.c_float, P, P, P, ALLREDUCE, P]
        L.orc_train_more.argtypes = [P, i32]
        L.orc_set_sampling.argtypes = [P, C.c_double, C.c_double, C.c_double, C.c_double, i64, u64]
        L.orc_free.argtypes = [P]
        L.orc_num_trees.argtypes = [P]
        L.orc_tree_size.argtypes = [P, i32]
        L.orc_tree.argtypes = [P, i32] + [P] * 9
        L.orc_margins.argtypes = [P, P]
        L.orc_predict.argtypes = [P, P, u64, u64, i32, i32, i32, i32, C.c_float, P]
        L.orc_scales.argtypes = [P, P]
        L.orc_model_cuts.argtypes = [P, P, P, P]
        L.orc_last_error.restype = C.c_char_p
        _lib = L
    return _lib


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


def default_threads() -> int:
    return max(1, len(os.sched_getaffinity(0)))


def dp_exp(x: float) -> float:
    return lib().orc_exp(float(x))


def cuts(x: np.ndarray, max_bin: int = 256, threads: int = 1, missing: float | None = None):
    x = np.ascontiguousarray(x, dtype=np.float32)
    R, F = x.shape
    cut = np.zeros((F, 256), np.float32)
    nb = np.zeros(F, np.uint16)
    hm = np.zeros(F, np.uint8)
    lib().orc_cuts(_p(x), R, F, F, max_bin, int(missing is not None), float(missing or 0.0), _p(cut), _p(nb),
                   _p(hm), threads)
    return cut, nb, hm


def radix_cuts(x: np.ndarray, max_bin: int = 256, allreduce=None, missing: float | None = None):
    """Cuts by the radix-selection search (the GPU algorithm) over this rank's
    rows; `allreduce(buf: np.ndarray[int64], op: int)` sums / maxes in place
    over all ranks (None: one rank)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    R, F = x.shape
    cut = np.zeros((F, 256), np.float32)
    nb = np.zeros(F, np.uint16)
    hm = np.zeros(F, np.uint8)
    cb = _callback(allreduce)
    lib().orc_radix_cuts(_p(x), R, F, F, max_bin, int(missing is not None), float(missing or 0.0), _p(cut), _p(nb),
                         _p(hm), cb, None)
    return cut, nb, hm


def _callback(allreduce):
    if allreduce is None:
        return ALLREDUCE()
    def fn(buf, n, op, ctx):
        allreduce(np.ctypeslib.as_array(buf, shape=(n,)), op)
    return ALLREDUCE(fn)


def bin_matrix(x: np.ndarray, cut, nb, hm, threads: int = 1, missing: float | None = None) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    R, F = x.shape
    stride = (F + 15) // 16 * 16
    bins = np.zeros((R, stride), np.uint8)
    lib().orc_bin_matrix(_p(x), R, F, F, _p(cut), _p(nb), _p(hm), int(missing is not None), float(missing or 0.0),
                         _p(bins), stride, threads)
    return bins


def gradients(objective: str, margin: np.ndarray, label: np.ndarray, threads: int = 1) -> np.ndarray:
    """Returns gh [K][R][2] float32."""
    margin = np.ascontiguousarray(margin, dtype=np.float32)
    label = np.ascontiguousarray(label, dtype=np.float32)
    R = label.shape[0]
    K = margin.size // R
    gh = np.zeros((K, R, 2), np.float32)
    lib().orc_gradients(OBJECTIVES[objective], K, _p(margin), _p(label), R, _p(gh), threads)
    return gh


def quantizer(gh_k: np.ndarray):
    gh_k = np.ascontiguousarray(gh_k, dtype=np.float32)
    sg = np.zeros(1, np.float32)
    sh = np.zeros(1, np.float32)
    lib().orc_quantizer(_p(gh_k), gh_k.shape[0], _p(sg), _p(sh))
    return float(sg[0]), float(sh[0])


def histograms(bins: np.ndarray, F: int, ghp: np.ndarray, ridx: np.ndarray, seg_begin, seg_end, sg: float,
               sh: float, threads: int = 1) -> np.ndarray:
    """hist[N][F][256][2] int64 over position segments [seg_begin, seg_end)."""
    bins = np.ascontiguousarray(bins, dtype=np.uint8)
    ghp = np.ascontiguousarray(ghp, dtype=np.float32)
    ridx = np.ascontiguousarray(ridx, dtype=np.uint32)
    sb = np.ascontiguousarray(seg_begin, dtype=np.int64)
    se = np.ascontiguousarray(seg_end, dtype=np.int64)
    out = np.zeros((len(sb), F, 256, 2), np.int64)
    lib().orc_histograms(_p(bins), bins.shape[1], F, _p(ghp), _p(ridx), _p(sb), _p(se), len(sb), sg, sh,
                         _p(out), threads)
    return out


def best_splits(hist: np.ndarray, nb, hm, totals: np.ndarray, sg: float, sh: float, lam=1.0, alpha=0.0,
                gamma=0.0, mcw=1.0):
    hist = np.ascontiguousarray(hist, dtype=np.int64)
    N, F = hist.shape[0], hist.shape[1]
    totals = np.ascontiguousarray(totals, dtype=np.int64)
    nb = np.ascontiguousarray(nb, dtype=np.uint16)
    hm = np.ascontiguousarray(hm, dtype=np.uint8)
    oi = np.zeros((N, 4), np.int32)
    og = np.zeros(N, np.float64)
    ol = np.zeros((N, 2), np.int64)
    lib().orc_best_splits(_p(hist), N, F, _p(nb), _p(hm), _p(totals), sg, sh, lam, alpha, gamma, mcw, _p(oi),
                          _p(og), _p(ol))
    return oi, og, ol


class Model:
    """Oracle training run; trees as dicts of numpy arrays."""

    def __init__(self, x: np.ndarray, y: np.ndarray, objective: str = "reg:squarederror", num_class: int = 1,
                 max_depth: int = 6, max_bin: int = 256, eta: float = 0.3, reg_lambda: float = 1.0,
                 alpha: float = 0.0, gamma: float = 0.0, min_child_weight: float = 1.0, base_margin: float = 0.0,
                 rounds: int = 1, threads: int = 1, subtract: bool = True, subsample: float = 1.0,
                 colsample_bytree: float = 1.0, colsample_bylevel: float = 1.0, colsample_bynode: float = 1.0,
                 seed: int = 0):
        self.x = np.ascontiguousarray(x, dtype=np.float32)
        self.y = np.ascontiguousarray(y, dtype=np.float32)
        R, F = self.x.shape
        self.R, self.F = R, F
        K = num_class if objective.startswith("multi:") else 1
        self.K = K
        self.objective = objective
        sampling = (subsample, colsample_bytree, colsample_bylevel, colsample_bynode) != (1.0, 1.0, 1.0, 1.0)
        self.h = lib().orc_train(_p(self.x), R, F, F, _p(self.y), OBJECTIVES[objective], K, max_depth, max_bin,
                                 eta, reg_lambda, alpha, gamma, min_child_weight, base_margin,
                                 0 if sampling else rounds, threads, int(subtract))
        if not self.h:
            raise RuntimeError(lib().orc_last_error().decode())
        if sampling:
            lib().orc_set_sampling(self.h, subsample, colsample_bytree, colsample_bylevel, colsample_bynode, seed, 0)
            lib().orc_train_more(self.h, rounds)

    @classmethod
    def sharded(cls, x: np.ndarray, y: np.ndarray, allreduce, objective: str = "reg:squarederror",
                num_class: int = 1, max_depth: int = 6, max_bin: int = 256, eta: float = 0.3, reg_lambda: float = 1.0,
                alpha: float = 0.0, gamma: float = 0.0, min_child_weight: float = 1.0, base_margin: float = 0.0,
                rounds: int = 1, threads: int = 1) -> "Model":
        """Training over this rank's rows; `allreduce(buf, op)` combines int64
        buffers over the ranks in place (op 0 = sum, 1 = max)."""
        self = cls.__new__(cls)
        self.x = np.ascontiguousarray(x, dtype=np.float32)
        self.y = np.ascontiguousarray(y, dtype=np.float32)
        R, F = self.x.shape
        self.R, self.F = R, F
        K = num_class if objective.startswith("multi:") else 1
        self.K = K
        self.objective = objective
        self._cb = _callback(allreduce)
        self.h = lib().orc_train_sharded(_p(self.x), R, F, F, _p(self.y), OBJECTIVES[objective], K, max_depth,
                                         max_bin, eta, reg_lambda, alpha, gamma, min_child_weight, base_margin,
                                         rounds, threads, self._cb, None)
        if not self.h:
            raise RuntimeError(lib().orc_last_error().decode())
        return self

    def __del__(self):
        # at interpreter exit the module globals may already be gone
        if getattr(self, "h", None) and lib is not None:
            lib().orc_free(self.h)
            self.h = None

    def train_more(self, rounds: int) -> None:
        lib().orc_train_more(self.h, rounds)

    def num_trees(self) -> int:
        return lib().orc_num_trees(self.h)

    def tree(self, t: int) -> dict:
        n = lib().orc_tree_size(self.h, t)
        out = {
            "left_children": np.zeros(n, np.int32), "right_children": np.zeros(n, np.int32),
            "split_indices": np.zeros(n, np.int32), "split_conditions": np.zeros(n, np.float32),
            "default_left": np.zeros(n, np.uint8), "base_weights": np.zeros(n, np.float32),
            "loss_changes": np.zeros(n, np.float32), "sum_hessian": np.zeros(n, np.float32),
            "split_bins": np.zeros(n, np.int32),
        }
        keys = ["left_children", "right_children", "split_indices", "split_conditions", "default_left",
                "base_weights", "loss_changes", "sum_hessian", "split_bins"]
        lib().orc_tree(self.h, t, *[_p(out[k]) for k in keys])
        return out

    def predict(self, x: np.ndarray, margin: bool = False, iteration_begin: int = 0, iteration_end: int = 0,
                missing: float = float("nan"), objective: str = None) -> np.ndarray:
        """Predictions of the trained ensemble: margins [R, K] (margin=True) or
        the objective's output ([R, K] probabilities for softprob, else [R]).
        The transform is the trained model's objective; `objective` only
        states it and must agree."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        R = x.shape[0]
        if objective is not None and objective != self.objective:
            raise ValueError(f"model objective is {self.objective}, not {objective}")
        softprob = self.objective == "multi:softprob"
        width = self.K if (margin or softprob) else 1
        out = np.zeros((R, width), np.float32)
        has_mv = not np.isnan(missing)
        rc = lib().orc_predict(self.h, _p(x), R, x.shape[1], 1 if margin else 0, iteration_begin, iteration_end,
                               int(has_mv), C.c_float(0.0 if not has_mv else missing), _p(out))
        if rc != 0:
            raise RuntimeError(lib().orc_last_error().decode())
        return out

    def margins(self) -> np.ndarray:
        m = np.zeros((self.R, self.K), np.float32)
        lib().orc_margins(self.h, _p(m))
        return m

    def scales(self) -> np.ndarray:
        s = np.zeros((self.num_trees(), 2), np.float32)
        lib().orc_scales(self.h, _p(s))
        return s

    def cuts(self):
        cut = np.zeros((self.F, 256), np.float32)
        nb = np.zeros(self.F, np.uint16)
        hm = np.zeros(self.F, np.uint8)
        lib().orc_model_cuts(self.h, _p(cut), _p(nb), _p(hm))
        return cut, nb, hm
