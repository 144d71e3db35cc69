"""Per-kernel parity of the CUDA path against the CPU oracle, through the
C-ABI kernel entry points.  Every comparison is bit-exact: cuts and bins are
order statistics, gradients use the same IEEE operation sequence, histograms
are integer sums of the same quantised values, and split gains are the same
double-precision expression."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


_alive = []


def cuda(a):
    """Device copy kept alive for the rest of the test session: the C-ABI
    receives raw pointers, so a temporary must not return to torch's caching
    allocator before the call has finished."""
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    _alive.append(t)
    return t


def ptr(t):
    return t.data_ptr()


@pytest.fixture(autouse=True)
def _release_buffers():
    yield
    torch.cuda.synchronize()
    _alive.clear()


def special_matrix(R, F, seed, nan_frac=0.0):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((R, F)).astype(np.float32)
    if F > 1:
        x[:, 1] = rng.integers(0, 5, R).astype(np.float32)           # few distinct values
    if F > 2:
        x[:, 2] = 3.0                                                 # constant column
    if F > 3:
        x[:, 3] = np.where(rng.random(R) < 0.5, -0.0, 0.0)            # signed zeros only
        x[: R // 3, 3] = rng.standard_normal(R // 3)
    if F > 4:
        x[:, 4] = rng.integers(0, 256, R).astype(np.float32)          # exactly 256 distinct values
    if F > 5:
        x[:, 5] = np.nan                                              # all missing
    if F > 6:
        x[:, 6] = rng.integers(0, 255, R).astype(np.float32)          # 255 distinct + missing below
        x[rng.random(R) < 0.1, 6] = np.nan
    if F > 7:
        x[:, 7] = np.round(rng.standard_normal(R) * 4) / 4            # heavy ties
    if nan_frac:
        mask = rng.random((R, F)) < nan_frac
        x[mask] = np.nan
    return x


def gpu_cuts(dp, x, max_bin):
    R, F = x.shape
    xd = cuda(x)
    cut = torch.zeros((F, 256), dtype=torch.float32, device="cuda")
    nb = torch.zeros(F, dtype=torch.int16, device="cuda")
    hm = torch.zeros(F, dtype=torch.uint8, device="cuda")
    dp.check(dp.lib().dp_quantile_cuts(ptr(xd), R, F, F, max_bin, ptr(cut), ptr(nb), ptr(hm), None))
    torch.cuda.synchronize()
    return cut.cpu().numpy(), nb.cpu().numpy().view(np.uint16), hm.cpu().numpy()


@pytest.mark.parametrize("R,F,max_bin,nan_frac,seed", [
    (1, 3, 256, 0.0, 0), (7, 9, 256, 0.0, 1), (1000, 9, 256, 0.0, 2), (5000, 12, 256, 0.05, 3),
    (20000, 16, 256, 0.0, 4), (20000, 9, 16, 0.0, 5), (3000, 40, 64, 0.2, 6), (70000, 33, 256, 0.01, 7),
])
def test_cuts_and_bins_match_oracle(dp, orc, R, F, max_bin, nan_frac, seed):
    x = special_matrix(R, F, seed, nan_frac)
    cut, nb, hm = gpu_cuts(dp, x, max_bin)
    ocut, onb, ohm = orc.cuts(x, max_bin, threads=4)
    np.testing.assert_array_equal(nb, onb)
    np.testing.assert_array_equal(hm, ohm)
    np.testing.assert_array_equal(cut.view(np.uint32), ocut.view(np.uint32))
    assert (nb <= max_bin).all()
    stride = (F + 15) // 16 * 16
    bins = torch.zeros((R, stride), dtype=torch.uint8, device="cuda")
    dp.check(dp.lib().dp_bin_matrix(ptr(cuda(x)), R, F, F, ptr(cuda(cut)), ptr(cuda(nb.view(np.int16))),
                                    ptr(bins), stride, None))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bins.cpu().numpy(), orc.bin_matrix(x, ocut, onb, ohm, threads=4))


def test_uint8_columns_get_one_bin_per_value(dp, orc):
    rng = np.random.default_rng(11)
    x = np.where(rng.random((6000, 20)) < 0.8, 0, rng.integers(1, 256, (6000, 20))).astype(np.float32)
    cut, nb, hm = gpu_cuts(dp, x, 256)
    distinct = np.array([len(np.unique(x[:, f])) for f in range(20)])
    np.testing.assert_array_equal(nb, distinct)
    assert not hm.any()


@pytest.mark.parametrize("objective,K", [("reg:squarederror", 1), ("binary:logistic", 1), ("multi:softprob", 4),
                                         ("multi:softmax", 10)])
def test_gradients_and_scales_match_oracle(dp, orc, objective, K):
    rng = np.random.default_rng(K)
    R = 30001
    margin = (rng.standard_normal((R, K)) * 3).astype(np.float32)
    if objective == "binary:logistic":
        y = rng.integers(0, 2, R).astype(np.float32)
    elif K > 1:
        y = rng.integers(0, K, R).astype(np.float32)
    else:
        y = rng.standard_normal(R).astype(np.float32)
    gh = torch.zeros((K, R, 2), dtype=torch.float32, device="cuda")
    sc = torch.zeros((K, 2), dtype=torch.float32, device="cuda")
    dp.check(dp.lib().dp_gradients(dp.OBJECTIVE_IDS[objective], K, ptr(cuda(margin)), ptr(cuda(y)), R, ptr(gh),
                                   ptr(sc), None))
    ogh = orc.gradients(objective, margin, y, threads=4)
    np.testing.assert_array_equal(gh.cpu().numpy().view(np.uint32), ogh.view(np.uint32))
    scales = sc.cpu().numpy()
    for k in range(K):
        assert tuple(scales[k]) == orc.quantizer(ogh[k])


@pytest.mark.parametrize("F,nodes,seed,nbins,R", [(32, 1, 0, 256, 40000), (16, 3, 1, 256, 40000),
                                                 (64, 5, 2, 256, 40000), (100, 2, 3, 256, 40000),
                                                 (784, 2, 4, 256, 40000), (32, 1, 5, 64, 200000),
                                                 (40, 4, 6, 16, 100000), (32, 2, 7, 256, 600000),
                                                 # 16- and 64-bin codes through the 256-bin kernel, which
                                                 # builds one segment and 512 or more
                                                 (24, 0, 8, 16, 150000), (32, 600, 9, 64, 300000)])
def test_histograms_match_oracle(dp, orc, F, nodes, seed, nbins, R):
    rng = np.random.default_rng(seed)
    stride = (F + 15) // 16 * 16
    bins = rng.integers(0, nbins, (R, stride)).astype(np.uint8)
    bins[:, F:] = 0
    gh = np.stack([rng.standard_normal(R), rng.random(R)], 1).astype(np.float32)
    ridx = rng.permutation(R).astype(np.uint32)
    # ragged segments incl. an empty one and one larger than a window
    cuts = np.sort(rng.choice(np.arange(1, R), nodes, replace=False))
    edges = np.concatenate([[0], cuts, [R]])
    sb = list(edges[:-1]) + [edges[1]]
    se = list(edges[1:]) + [edges[1]]
    sg, sh = orc.quantizer(gh)
    hist = torch.zeros((len(sb), F, 256, 2), dtype=torch.int64, device="cuda")
    sbn = np.array(sb, np.int64)
    sen = np.array(se, np.int64)
    dp.check(dp.lib().dp_hist_build(ptr(cuda(bins)), stride, F, nbins, ptr(cuda(gh)), ptr(cuda(ridx)), sbn.ctypes.data,
                                    sen.ctypes.data, len(sb), sg, sh, ptr(hist), None))
    ohist = orc.histograms(bins, F, gh, ridx, sb, se, sg, sh, threads=4)
    np.testing.assert_array_equal(hist.cpu().numpy(), ohist)
    assert (ohist[-1] == 0).all()


@pytest.mark.parametrize("wide", ["0", "1"])
@pytest.mark.parametrize("F,nodes,chunk", [(64, 1, 0), (100, 3, 40000), (160, 2, 70000), (40, 5, 0)])
def test_both_256_bin_kernels_with_long_tasks(dp, orc, monkeypatch, wide, F, nodes, chunk):
    """The 32- and 64-feature 256-bin kernels (DP_HIST_WIDE; the latter keeps
    its window sums in tensor memory) on tasks long enough to fold several
    16383-row windows (DP_HIST_MIN_CHUNK), with partial last tiles, a feature
    count above one tile, nodes split into pieces (drained with atomics) and
    nodes built whole (drained with stores)."""
    monkeypatch.setenv("DP_HIST_WIDE", wide)
    if chunk:
        monkeypatch.setenv("DP_HIST_MIN_CHUNK", str(chunk))
    R = 150000
    rng = np.random.default_rng(40 + F)
    stride = (F + 15) // 16 * 16
    bins = rng.integers(0, 256, (R, stride)).astype(np.uint8)
    bins[:, F:] = 0
    gh = np.stack([rng.standard_normal(R), rng.random(R)], 1).astype(np.float32)
    ridx = rng.permutation(R).astype(np.uint32)
    cuts = np.sort(rng.choice(np.arange(1, R), nodes - 1, replace=False)) if nodes > 1 else np.array([], np.int64)
    edges = np.concatenate([[0], cuts, [R]]).astype(np.int64)
    sb, se = np.ascontiguousarray(edges[:-1]), np.ascontiguousarray(edges[1:])
    sg, sh = orc.quantizer(gh)
    hist = torch.zeros((len(sb), F, 256, 2), dtype=torch.int64, device="cuda")
    dp.check(dp.lib().dp_hist_build(ptr(cuda(bins)), stride, F, 256, ptr(cuda(gh)), ptr(cuda(ridx)), sb.ctypes.data,
                                    se.ctypes.data, len(sb), sg, sh, ptr(hist), None))
    np.testing.assert_array_equal(hist.cpu().numpy(), orc.histograms(bins, F, gh, ridx, sb, se, sg, sh, threads=4))


@pytest.mark.parametrize("lam,alpha,gamma,mcw,nan_frac", [(1.0, 0.0, 0.0, 1.0, 0.0), (2.0, 0.5, 0.3, 5.0, 0.1),
                                                          (0.0, 0.0, 0.0, 0.0, 0.3), (1.0, 2.0, 0.0, 0.1, 0.0)])
def test_split_evaluation_matches_oracle(dp, orc, lam, alpha, gamma, mcw, nan_frac):
    rng = np.random.default_rng(5)
    R, F = 20000, 24
    x = special_matrix(R, F, 9, nan_frac)
    y = (np.nan_to_num(x[:, 0]) + 0.3 * rng.standard_normal(R) > 0).astype(np.float32)
    cut, nb, hm = orc.cuts(x, 256, threads=4)
    bins = orc.bin_matrix(x, cut, nb, hm, threads=4)
    margin = np.zeros((R, 1), np.float32)
    gh = orc.gradients("binary:logistic", margin, y)[0]
    sg, sh = orc.quantizer(gh)
    ridx = np.arange(R, dtype=np.uint32)
    edges = [0, 5, 333, 9000, 9001, R]
    hist = orc.histograms(bins, F, gh, ridx, edges[:-1], edges[1:], sg, sh, threads=4)
    totals = hist[:, 0, :, :].sum(axis=1)
    oi, og, ol = orc.best_splits(hist, nb, hm, totals, sg, sh, lam, alpha, gamma, mcw)
    N = hist.shape[0]
    gi = np.zeros((N, 4), np.int32)
    gg = np.zeros(N, np.float64)
    gl = np.zeros((N, 2), np.int64)
    dp.check(dp.lib().dp_eval_splits(ptr(cuda(hist)), N, F, ptr(cuda(nb.view(np.int16))), ptr(cuda(hm)),
                                     np.ascontiguousarray(totals).ctypes.data, sg, sh, lam, alpha, gamma, mcw,
                                     gi.ctypes.data, gg.ctypes.data, gl.ctypes.data))
    np.testing.assert_array_equal(gi[:, 3], oi[:, 3])
    valid = oi[:, 3] == 1
    np.testing.assert_array_equal(gi[valid], oi[valid])
    np.testing.assert_array_equal(gg[valid].view(np.uint64), og[valid].view(np.uint64))
    np.testing.assert_array_equal(gl[valid], ol[valid])


@pytest.mark.parametrize("F,nodes,nbins,R", [(32, 1, 256, 1_500_000), (128, 3, 256, 300_000), (48, 9, 64, 400_000)])
def test_quantized_histogram_plan_matches_oracle(dp, orc, F, nodes, nbins, R):
    """The engine's layout: int32 (g, h) pairs from dp_quantize_gh, tasks from a
    prepared plan, many tasks per node and several accumulation windows."""
    import ctypes
    rng = np.random.default_rng(F + nodes)
    stride = (F + 15) // 16 * 16
    bins = rng.integers(0, nbins, (R, stride)).astype(np.uint8)
    gh = np.stack([rng.standard_normal(R), rng.random(R)], 1).astype(np.float32)
    ridx = rng.permutation(R).astype(np.uint32)
    edges = np.concatenate([[0], np.sort(rng.choice(np.arange(1, R), nodes - 1, replace=False)), [R]]).astype(np.int64)
    sb, se = np.ascontiguousarray(edges[:-1]), np.ascontiguousarray(edges[1:])
    sg, sh = orc.quantizer(gh)
    ghd = cuda(gh)
    dp.check(dp.lib().dp_quantize_gh(ptr(ghd), R, sg, sh, None))
    q = ghd.cpu().numpy().view(np.int32)
    np.testing.assert_array_equal(q[:, 0], np.rint(gh[:, 0] * np.float32(sg)).astype(np.int32))
    hist = torch.empty((nodes, F, 256, 2), dtype=torch.int64, device="cuda")
    plan = ctypes.c_void_p()
    binsd, ridxd = cuda(bins), cuda(ridx)
    dp.check(dp.lib().dp_hist_prepare(ptr(binsd), stride, F, nbins, 1, ptr(ghd), ptr(ridxd), sb.ctypes.data,
                                      se.ctypes.data, nodes, sg, sh, ptr(hist), ctypes.byref(plan)))
    for _ in range(2):  # reruns must give the same result (the plan re-zeroes its output)
        dp.check(dp.lib().dp_hist_run(plan, None))
    torch.cuda.synchronize()
    dp.check(dp.lib().dp_hist_free(plan))
    ohist = orc.histograms(bins, F, gh, ridx, sb, se, sg, sh, threads=8)
    np.testing.assert_array_equal(hist.cpu().numpy(), ohist)
