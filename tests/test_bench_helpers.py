"""CPU checks of bench.py's helpers: the synthetic CSV of the ingest
measurement is a table the reference's own decoder accepts (oracle/_ref/ref_csv,
built from native/decision_programs_csv.hpp), and the per-level breakdown reads
the profiler's launch log in order."""
import json
import pathlib
import subprocess
import sys

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
REF = ROOT / "oracle" / "_ref" / "ref_csv"
sys.path.insert(0, str(ROOT))


@pytest.mark.skipif(not REF.exists(), reason="reference CSV harness not built (needs the reference sources)")
def test_bench_csv_is_accepted_by_the_reference_decoder(tmp_path):
    import bench
    data = bench.csv_text(3000, 7, seed=5)
    src = tmp_path / "b.csv"
    src.write_bytes(data)
    subprocess.run([str(REF), str(src), "label", "auto", str(tmp_path)], check=True, timeout=120)
    assert not (tmp_path / "error.txt").exists()
    meta = json.loads((tmp_path / "meta.json").read_text())
    assert (meta["rows"], meta["features"], meta["classes"], meta["header"]) == (3000, 7, 10, True)
    values = np.fromfile(tmp_path / "values.f32", dtype="<f4").reshape(3000, 7)
    # fixed-width decimals with four places, |v| < 1000
    assert np.all(np.abs(values) < 1000) and np.allclose(values * 1e4, np.rint(values * 1e4), atol=0.05)


def test_per_level_reads_the_launch_log():
    import bench
    log = [["gradients", 1.0, 0], ["histograms", 2.0, 0], ["eval_splits", 0.5, 0], ["partition", 0.25, 0],
           ["histograms", 1.5, 0], ["exchange_hist", 0.75, 0], ["partition", 0.1, 0], ["leaf_update", 0.2, 0],
           ["gradients", 1.0, 0], ["histograms", 3.0, 0], ["partition", 0.3, 0], ["leaf_update", 0.4, 0]]
    levels = bench.per_level(log)
    assert levels == [{"histograms": 3.0, "partition": 0.3, "leaf_update": 0.4}]
    assert bench.per_level(log[:8]) == [{"histograms": 2.0, "eval_splits": 0.5, "partition": 0.25},
                                        {"histograms": 1.5, "exchange_hist": 0.75, "partition": 0.1,
                                         "leaf_update": 0.2}]


def test_sklearn_leg_reports_time_per_tree(monkeypatch):
    pytest.importorskip("sklearn")
    import bench
    monkeypatch.setattr(bench, "SKLEARN_ROWS", 4000)
    monkeypatch.setattr(bench, "SKLEARN_TREES", 2)
    rng = np.random.default_rng(3)
    x = rng.standard_normal((6000, 8)).astype(np.float32)
    y = (x[:, 0] + 0.1 * rng.standard_normal(6000)).astype(np.float32)
    out = bench.sklearn_leg(x, y, 2)
    assert out["unit"] == "rows*trees/s" and out["cores"] == 2
    assert out["value"] > 0 and out["seconds_per_tree"] > 0
    assert "4000 rows" in out["sample"] and out["impl"].startswith("scikit-learn")
