"""Accuracy of the quantised histogram sums against exact sums of the fp32
(g, h) pairs.

Histograms hold exact int64 sums of q = rint(v * s), so they do not depend on
summation order, block count or rank count (the GPU kernels equal the CPU
oracle bit for bit, tests/test_gpu_kernels.py).  What quantising costs is
accuracy: each row's value moves by at most 0.5 / s, and the scale s is a
power of two that maps the round's largest |g| into [2^16, 2^17] and the
largest h into [2^17, 2^18].  These tests bound the dequantised sums
Σq / s against fp64 sums of the same fp32 values, per (feature, bin) cell:
  * always: |Σq/s − Σv| <= n * 0.5 / s  (n = rows in the cell);
  * hessian sums (h >= 0): relative error below 1e-5 (the figure the north
    star gives for fp32 histogram sums);
  * gradient sums, whose terms cancel: error below 1e-5 of Σ|g| (relative to
    |Σg| itself the error is unbounded when the sum is near zero).
"""
import numpy as np
import pytest


def case(kind, rng, R):
    if kind == "normal-uniform":  # config 5's (g, h) ~ N(0,1) x U(0,1)
        return rng.standard_normal(R), rng.random(R)
    m = 2.0 * rng.standard_normal(R)
    if kind == "logistic":
        y = rng.random(R) < 1.0 / (1.0 + np.exp(-m))
        p = 1.0 / (1.0 + np.exp(-m))
        return p - y, np.maximum(p * (1.0 - p), 1e-16)
    if kind == "squared-error":
        return m - rng.standard_normal(R), np.ones(R)
    raise ValueError(kind)


@pytest.mark.parametrize("kind", ["normal-uniform", "logistic", "squared-error"])
def test_quantised_sums_against_fp64(orc, kind):
    rng = np.random.default_rng({"normal-uniform": 1, "logistic": 2, "squared-error": 3}[kind])
    R, F = 300_000, 4
    bins = rng.integers(0, 256, (R, 16)).astype(np.uint8)
    g, h = case(kind, rng, R)
    gh = np.stack([g, h], 1).astype(np.float32)
    sg, sh = orc.quantizer(gh)
    hist = orc.histograms(bins, F, gh, np.arange(R, dtype=np.uint32), [0], [R], sg, sh,
                          threads=orc.default_threads())[0]
    g64, h64 = gh[:, 0].astype(np.float64), gh[:, 1].astype(np.float64)
    for f in range(F):
        b = bins[:, f]
        n = np.bincount(b, None, 256)
        eg, eh = np.bincount(b, g64, 256), np.bincount(b, h64, 256)
        ag = np.bincount(b, np.abs(g64), 256)
        qg, qh = hist[f, :, 0] / sg, hist[f, :, 1] / sh
        # the per-row rounding bound, summed over the cell
        assert np.all(np.abs(qg - eg) <= n * 0.5 / sg + 1e-9)
        assert np.all(np.abs(qh - eh) <= n * 0.5 / sh + 1e-9)
        full = n >= 100
        assert full.sum() == 256
        assert np.max(np.abs(qh - eh)[full] / eh[full]) < 1e-5
        assert np.max(np.abs(qg - eg)[full] / ag[full]) < 1e-5
