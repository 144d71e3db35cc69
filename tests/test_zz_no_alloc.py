"""dp_hist_build_noalloc: the histogram build for callers that cannot
allocate device memory (a pre-reserved memory pool, or a path that must not
call cudaMalloc/cudaFree).  Its result must equal dp_hist_build's, the
allocating entry point, exactly (integer sums), on consecutive calls that
reuse its fixed scratch array, and both must equal the CPU oracle's sums;
it must refuse work above its capacity.
This file is collected last and depends on nothing the other tests set up."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def make_case(seed, R, F, nbins, nseg):
    rng = np.random.default_rng(seed)
    stride = (F + 15) // 16 * 16
    bins = rng.integers(0, nbins, (R, stride)).astype(np.uint8)
    bins[:, F:] = 0
    gh = np.stack([rng.standard_normal(R), rng.random(R)], 1).astype(np.float32)
    ridx = rng.permutation(R).astype(np.uint32)
    cuts = np.sort(rng.choice(np.arange(1, R), nseg - 1, replace=False))
    edges = np.concatenate([[0], cuts, [R]]).astype(np.int64)
    sb = np.concatenate([edges[:-1], [edges[1]]]).astype(np.int64)  # plus one empty segment
    se = np.concatenate([edges[1:], [edges[1]]]).astype(np.int64)
    sg = float(np.ldexp(1.0, 17 - np.frexp(np.abs(gh[:, 0]).max())[1]))
    sh = float(np.ldexp(1.0, 18 - np.frexp(gh[:, 1].max())[1]))
    dev = {k: torch.from_numpy(v).cuda() for k, v in dict(bins=bins, gh=gh, ridx=ridx).items()}
    return dict(stride=stride, F=F, nbins=nbins, sb=sb, se=se, sg=sg, sh=sh, dev=dev,
                host=dict(bins=bins, gh=gh, ridx=ridx))


def run(dp, fn, c):
    hist = torch.full((len(c["sb"]), c["F"], 256, 2), -7, dtype=torch.int64, device="cuda")
    rc = fn(c["dev"]["bins"].data_ptr(), c["stride"], c["F"], c["nbins"], c["dev"]["gh"].data_ptr(),
            c["dev"]["ridx"].data_ptr(), c["sb"].ctypes.data, c["se"].ctypes.data, len(c["sb"]), c["sg"], c["sh"],
            hist.data_ptr(), None)
    dp.check(rc)
    torch.cuda.synchronize()
    return hist.cpu().numpy()


def test_noalloc_histogram_equals_the_allocating_entry_point(dp, orc):
    lib = dp.lib()
    a = make_case(1, 200_000, 64, 256, 3)
    b = make_case(2, 60_000, 20, 64, 6)
    want_a = run(dp, lib.dp_hist_build, a)
    want_b = run(dp, lib.dp_hist_build, b)
    assert want_a.any() and want_b.any()
    # the reference sums, from the CPU oracle, for both entry points
    for c, want in ((a, want_a), (b, want_b)):
        h = c["host"]
        np.testing.assert_array_equal(
            want, orc.histograms(h["bins"], c["F"], h["gh"], h["ridx"], c["sb"], c["se"], c["sg"], c["sh"], threads=4))
    # two calls in a row on different shapes, then the first shape again: the
    # shared scratch must carry nothing over from the previous call
    np.testing.assert_array_equal(run(dp, lib.dp_hist_build_noalloc, a), want_a)
    np.testing.assert_array_equal(run(dp, lib.dp_hist_build_noalloc, b), want_b)
    np.testing.assert_array_equal(run(dp, lib.dp_hist_build_noalloc, a), want_a)


def test_noalloc_refuses_work_above_its_capacity(dp):
    lib = dp.lib()
    R, F = 32769, 1  # 32769 one-row segments x 1 feature tile = 32769 tasks > 32768
    bins = torch.zeros((R, 16), dtype=torch.uint8, device="cuda")
    gh = torch.zeros((R, 2), dtype=torch.float32, device="cuda")
    ridx = torch.arange(R, dtype=torch.int32, device="cuda")
    sb = np.arange(R, dtype=np.int64)
    se = sb + 1
    # sized for the full request (134 MB), so the output stays in bounds
    # whatever happens; the call must refuse on the host, before device work
    hist = torch.empty((R, F, 256, 2), dtype=torch.int64, device="cuda")
    rc = lib.dp_hist_build_noalloc(bins.data_ptr(), 16, F, 256, gh.data_ptr(), ridx.data_ptr(), sb.ctypes.data,
                                   se.ctypes.data, R, 1.0, 1.0, hist.data_ptr(), None)
    assert rc == -1
    msg = lib.XGBGetLastError().decode()
    assert "capacity of 32768" in msg and "32769" in msg
