"""Freed boosters and matrices hand their device memory to the library's slab
cache (csrc/common.h, SlabCache), and later ones reuse it without zeroing: the
models trained on reused memory must be bit-identical to the first, also
after dp_release_cached_memory() has freed what was kept."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def fit(dp, x, y, params, rounds):
    d = dp.DMatrix.from_host(x, y)
    b = dp.train(params, d, rounds)
    raw = b.save_raw()
    margins = b.margins(len(x), 1)
    b.free()
    d.free()
    return raw, margins


def test_models_on_reused_memory_are_identical(dp):
    rng = np.random.default_rng(8)
    x = rng.standard_normal((30_000, 20)).astype(np.float32)
    x[rng.random(x.shape) < 0.03] = np.nan
    y = (np.nan_to_num(x[:, 0]) * np.nan_to_num(x[:, 1]) + 0.2 * rng.standard_normal(30_000) > 0).astype(np.float32)
    params = {"objective": "binary:logistic", "tree_method": "hist", "device": "cuda:0", "max_depth": 6}
    first, m1 = fit(dp, x, y, params, 4)
    # a smaller job in between leaves its memory in the cache as well
    fit(dp, x[:5000], y[:5000], params | {"max_depth": 3}, 2)
    again, m2 = fit(dp, x, y, params, 4)  # matrix and booster memory reused
    assert again == first
    assert dp.lib().dp_release_cached_memory() == 0
    fresh, m3 = fit(dp, x, y, params, 4)  # allocated anew
    assert fresh == first
    np.testing.assert_array_equal(m1.view(np.uint32), m2.view(np.uint32))
    np.testing.assert_array_equal(m1.view(np.uint32), m3.view(np.uint32))
