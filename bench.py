"""Benchmark of the GBDT-training hot path (BASELINE config 4 as the step).

A step is one boosting round of squared-error regression (one depth-10 tree)
over 10,000,000 rows x 128 fp32 features binned to 256 uint8 bins, rows
sharded over the ranks (strong scaling: the total row count is fixed).  The
target is a seeded random depth-6, 20-tree ensemble plus N(0, 0.1) noise.
Data is synthetic (seeded) with BASELINE's shapes and distributions.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

value    rows*trees/s of the timed rounds, inputs resident in HBM (device
         events around the rounds, max over ranks).
e2e      the same metric through the C-ABI with host inputs: pinned-host
         fp32 matrix and labels copied to the device, DMatrix creation (cuts
         and bins), W+K rounds, the model read back as JSON.
roofline histogram kernel: algorithmic bytes rows*(F + 12) + slots*F*256*16
         per launch over its CUDA-event duration on the library stream.
The reference arm (--impl reference) times the CPU oracle: the reference
repository trains only through an external GPU library that is absent here,
so the restatement of the same algorithm is the CPU implementation of the path.
cpu_third_party (one GPU, rank 0): scikit-learn's HistGradientBoostingRegressor
on a 2M-row sample of the same data, a tuned CPU library for context; it is not
the parity oracle.
"""
from __future__ import annotations

import argparse
import json
import re
import os
import pathlib
import statistics
import sys
import threading
import time

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "decision-programs_b200"))

ROWS = 10_000_000
FEATURES = 128
DEPTH = 10
CHUNK = 250_000           # generation unit; the dataset does not depend on the rank count
SEED = 20240601
PARAMS = {"objective": "reg:squarederror", "tree_method": "hist", "max_depth": DEPTH, "max_bin": 256, "eta": 0.3,
          "lambda": 1.0, "min_child_weight": 1.0}
WORKLOAD = "config4: reg:squarederror 10M x 128 fp32 -> 256 uint8 bins, depth 10, one tree per step"


def workload_config(rows: int = ROWS) -> dict:
    """The `config` object of both arms' lines.  It names the workload only,
    so the GPU arm and the reference arm report the same object for the same
    work; how each arm spreads it (GPUs or host threads) is the line's
    `parallelism`."""
    return {"workload": WORKLOAD, "rows": rows, "features": FEATURES, "max_depth": DEPTH, "max_bin": 256,
            "l2": "inputs (1.28 GB of bins, 5.1 GB fp32) exceed the 126 MB L2"}


def cpu_model() -> str:
    """The host CPU's model name (Linux /proc/cpuinfo), reported beside the
    thread count of every CPU figure."""
    try:
        for line in pathlib.Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text())
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "fallback": True}


# --------------------------------------------------------------------------- data
def teacher(seed: int = SEED):
    """Random depth-6 x 20-tree ensemble: feature, threshold per internal node,
    value per leaf."""
    rs = np.random.RandomState(seed)
    feats = rs.randint(0, FEATURES, (20, 63))
    thr = rs.normal(0.0, 0.7, (20, 63)).astype(np.float32)
    leaf = rs.normal(0.0, 1.0, (20, 64)).astype(np.float32)
    return feats, thr, leaf


def make_chunk(torch, c: int, device):
    g = torch.Generator(device=device)
    g.manual_seed(SEED * 1000 + c)
    x = torch.randn((CHUNK, FEATURES), device=device, generator=g, dtype=torch.float32)
    feats, thr, leaf = (torch.from_numpy(a).to(device) for a in teacher())
    y = torch.zeros(CHUNK, device=device)
    for t in range(20):
        idx = torch.zeros(CHUNK, dtype=torch.long, device=device)
        for _ in range(6):
            f = feats[t][idx]
            go = (x.gather(1, f[:, None])[:, 0] >= thr[t][idx]).long()
            idx = 2 * idx + 1 + go
        y += leaf[t][idx - 63]
    y += 0.1 * torch.randn(CHUNK, device=device, generator=g)
    return x, y


def shard(torch, rank: int, world: int, device, rows: int = ROWS):
    nchunks = rows // CHUNK
    mine = [c for c in range(nchunks) if c * world // nchunks == rank]
    xs, ys = zip(*(make_chunk(torch, c, device) for c in mine))
    return torch.cat(xs).contiguous(), torch.cat(ys).contiguous()


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """SM clock and clock-event reasons of one GPU, sampled every 100 ms from a
    background thread through NVML in this process (spawning nvidia-smi inside
    the timed region stalls the driver).  Falls back to nvidia-smi when NVML is
    unavailable."""

    def __init__(self, torch, device_index: int):
        self.torch = torch
        self.dev = device_index
        self.samples: list[tuple[float, float, int]] = []
        self._stop = threading.Event()
        self.nvml = None
        self.handle = None

    def _open(self):
        import pynvml
        pynvml.nvmlInit()
        props = self.torch.cuda.get_device_properties(self.dev)
        handle = None
        try:
            bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
            handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            handle = pynvml.nvmlDeviceGetHandleByIndex(self.dev)
        self.nvml, self.handle = pynvml, handle

    def _run(self):
        nv, h = self.nvml, self.handle
        mx = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        while not self._stop.is_set():
            try:
                self.samples.append((float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)), mx,
                                     int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))))
            except Exception:
                pass
            self._stop.wait(0.1)

    def start(self):
        try:
            self._open()
        except Exception:
            self.nvml = None
            return
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t.start()
        t0 = time.time()
        while not self.samples and time.time() - t0 < 2.0:
            time.sleep(0.01)

    def stop(self) -> dict:
        if self.nvml is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["NVML unavailable"], "samples": 0}
        self._stop.set()
        self.t.join(timeout=2)
        nv = self.nvml
        names = {"hw_slowdown": nv.nvmlClocksEventReasonHwSlowdown,
                 "hw_thermal_slowdown": nv.nvmlClocksEventReasonHwThermalSlowdown,
                 "sw_thermal_slowdown": nv.nvmlClocksEventReasonSwThermalSlowdown,
                 "sw_power_cap": nv.nvmlClocksEventReasonSwPowerCap}
        reasons = sorted({n for _, _, r in self.samples for n, bit in names.items() if r & bit})
        sm = [c for c, _, _ in self.samples]
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(m for _, m, _ in self.samples) if self.samples else None,
                "reasons": reasons, "samples": len(sm), "source": "NVML, 100 ms"}


# --------------------------------------------------------------------------- reference / CPU arm
def config4_host(torch, rows: int = ROWS):
    """The config-4 matrix and targets in host memory.  Generated with the
    same per-chunk seeds as the GPU arm; on a machine with a GPU the chunks
    are drawn on it (torch's CUDA generator), so both arms train on the same
    values, and copied back.  Returns (x, y, where)."""
    if torch.cuda.is_available():
        x, y = shard(torch, 0, 1, torch.device("cuda", 0), rows)
        xh, yh = x.cpu().numpy(), y.cpu().numpy()
        del x, y
        torch.cuda.empty_cache()
        return xh, yh, "drawn on the GPU, as the GPU arm's"
    x, y = shard(torch, 0, 1, "cpu", rows)
    return x.numpy(), y.numpy(), "drawn on the CPU (no GPU: same distribution, other draws)"


def oracle_model(x, y, threads: int):
    """The CPU oracle on the config-4 data, cuts and bins built, no tree yet."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    return oracle.Model(x, y, "reg:squarederror", max_depth=DEPTH, max_bin=256, eta=0.3, reg_lambda=1.0,
                        min_child_weight=1.0, rounds=0, threads=threads)


def reference_arm(args) -> None:
    """The CPU implementation of the path on the GPU arm's workload: the
    oracle trains depth-10 trees over all 10M x 128 rows of config 4, one tree
    per step, with every host thread; cuts and bins are built before the
    timed steps, as the GPU arm's are."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch
    threads = len(os.sched_getaffinity(0))
    x, y, where = config4_host(torch, ROWS)
    m = oracle_model(x, y, threads)
    for _ in range(args.warmup):
        m.train_more(1)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        m.train_more(1)
    dt = time.perf_counter() - t0
    value = ROWS * args.steps / dt
    line = {
        "impl": "reference", "metric": "boosting rows*trees/s (config 4 step, 1 tree)", "value": value,
        "unit": "rows*trees/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * dt / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u8 bins / int64 sums",
        "data": "synthetic (seeded)",
        "config": workload_config(ROWS),
        "parallelism": f"CPU oracle on {threads} host threads; every step one tree over all {ROWS} rows",
        "cpu_baseline": {"value": value, "unit": "rows*trees/s", "cores": threads, "cpu": cpu_model(),
                         "kind": "port",
                         "sample": f"the whole config-4 workload ({ROWS} rows x {FEATURES} features, data {where}), "
                                   f"one depth-10 tree per step, {args.steps} timed steps after {args.warmup} "
                                   f"warm-up trees (C++ oracle, {threads} threads)"},
        "e2e": {"value": value, "unit": "rows*trees/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# trees of the benchmarked run that are compared with the CPU oracle's
C4_PARITY_TREES = 3


def config4_cpu_leg(torch, first_trees: list[dict]) -> dict:
    """CPU baseline and full-size parity of the benchmarked workload: the
    oracle trains the first C4_PARITY_TREES trees over all 10M x 128 rows of
    the same data (drawn on the GPU with the same seeds), timed on every host
    thread, and its trees are compared field by field with the GPU run's."""
    threads = len(os.sched_getaffinity(0))
    x, y, where = config4_host(torch, ROWS)
    m = oracle_model(x, y, threads)
    t0 = time.perf_counter()
    m.train_more(C4_PARITY_TREES)
    dt = time.perf_counter() - t0
    same = same_trees(first_trees, m)
    del m
    third = sklearn_leg(x, y, threads)
    del x, y
    out = {"value": ROWS * C4_PARITY_TREES / dt, "unit": "rows*trees/s", "cores": threads, "cpu": cpu_model(),
           "kind": "port",
           "sample": f"the whole config-4 workload ({ROWS} rows, data {where}), the first {C4_PARITY_TREES} "
                     f"depth-10 trees (C++ oracle, {threads} threads, {dt:.1f} s; cuts and bins built before)",
           "trees_identical_to_oracle": same, "trees_compared": C4_PARITY_TREES}
    if third is not None:
        out["third_party"] = third
    return out


SKLEARN_ROWS = 2_000_000
SKLEARN_TREES = 4


def sklearn_leg(x, y, threads: int):
    """A tuned third-party CPU implementation of the same algorithm, for
    context beside the oracle: scikit-learn's HistGradientBoostingRegressor
    (histograms with sibling subtraction, depth-wise limit 10, lambda 1, eta
    0.3, 255 value bins) on the first SKLEARN_ROWS rows of the config-4 data.
    Binning is excluded: the time per tree is the difference between fits of
    1 + SKLEARN_TREES trees and of one tree.  It is not the parity oracle and
    its trees differ (its own binning and tie rules).  None when scikit-learn
    is not installed."""
    try:
        import sklearn
        from sklearn.ensemble import HistGradientBoostingRegressor
        from threadpoolctl import threadpool_limits
    except ImportError:
        return None
    xs, ys = np.ascontiguousarray(x[:SKLEARN_ROWS]), np.ascontiguousarray(y[:SKLEARN_ROWS])

    def fit(trees: int) -> float:
        h = HistGradientBoostingRegressor(max_iter=trees, max_depth=DEPTH, max_leaf_nodes=None, max_bins=255,
                                          learning_rate=0.3, l2_regularization=1.0, min_samples_leaf=1,
                                          early_stopping=False)
        t0 = time.perf_counter()
        h.fit(xs, ys)
        return time.perf_counter() - t0

    try:
        with threadpool_limits(limits=threads):
            t1 = fit(1)
            tn = fit(1 + SKLEARN_TREES)
    except Exception as e:  # context only: never cost the bench line
        return {"error": f"{type(e).__name__}: {e}"[:200]}
    per_tree = max(tn - t1, 1e-9) / SKLEARN_TREES
    return {"value": SKLEARN_ROWS / per_tree, "unit": "rows*trees/s", "cores": threads, "cpu": cpu_model(),
            "impl": f"scikit-learn {sklearn.__version__} HistGradientBoostingRegressor",
            "sample": f"first {SKLEARN_ROWS} rows of the config-4 data, depth-10 trees; time per tree = "
                      f"(fit of {1 + SKLEARN_TREES} trees - fit of 1) / {SKLEARN_TREES}, binning excluded",
            "seconds_per_tree": per_tree}


# --------------------------------------------------------------------------- configs 1-3
def c1_data(torch, device):
    """Config 1: 20,000 x 16 N(0,1); y = 1[x0 + 0.5 x1 x2 + N(0, 0.3) > 0]."""
    g = torch.Generator(device=device)
    g.manual_seed(SEED + 1)
    x = torch.randn((20_000, 16), device=device, generator=g)
    noise = 0.3 * torch.randn(20_000, device=device, generator=g)
    y = ((x[:, 0] + 0.5 * x[:, 1] * x[:, 2] + noise) > 0).float()
    return x.contiguous(), y


def c2_data(torch, device):
    """Config 2: 1,000,000 x 64 (32 columns N(0,1), 32 Uniform(0,1)); label =
    sign of a seeded sparse linear-plus-pairwise teacher (centred at its
    median), 10% of labels flipped."""
    R = 1_000_000
    g = torch.Generator(device=device)
    g.manual_seed(SEED + 2)
    x = torch.cat([torch.randn((R, 32), device=device, generator=g),
                   torch.rand((R, 32), device=device, generator=g)], 1).contiguous()
    rs = np.random.RandomState(SEED + 2)
    lin = rs.choice(64, 12, replace=False)
    w = rs.normal(0.0, 1.0, 12)
    pairs = rs.choice(64, (6, 2))
    c = rs.normal(0.0, 1.0, 6)
    score = torch.zeros(R, device=device)
    for f, wf in zip(lin, w):
        score += float(wf) * x[:, int(f)]
    for (i, j), cf in zip(pairs, c):
        score += float(cf) * x[:, int(i)] * x[:, int(j)]
    y = (score > score.median()).float()
    flip = torch.rand(R, device=device, generator=g) < 0.1
    y = torch.where(flip, 1.0 - y, y)
    return x, y.contiguous()


def c3_data(torch, device):
    """Config 3 (MNIST-shaped, synthetic): 60,000 x 784 uint8 values, 80%
    zeros, non-zeros Uniform{1..255}; 10 classes = argmax of a seeded linear
    teacher on the features.  Values go in as fp32 (integers 0..255)."""
    R, F = 60_000, 784
    g = torch.Generator(device=device)
    g.manual_seed(SEED + 3)
    nz = torch.rand((R, F), device=device, generator=g) < 0.2
    v = torch.randint(1, 256, (R, F), device=device, generator=g).float()
    x = torch.where(nz, v, torch.zeros((), device=device)).contiguous()
    w = torch.randn((F, 10), device=device, generator=g)
    y = torch.argmax(x @ w, 1).float().contiguous()
    return x, y


CONFIGS = [
    ("config1", c1_data, {"objective": "binary:logistic", "max_depth": 4}, 20, 1),
    ("config2", c2_data, {"objective": "binary:logistic", "max_depth": 8}, 100, 1),
    ("config3", c3_data, {"objective": "multi:softprob", "num_class": 10, "max_depth": 6}, 50, 10),
]
# rounds of each config that the CPU oracle trains, timed and compared tree by
# tree with the GPU run's first rounds (configs 1 and 2 in full)
CPU_ROUNDS = {"config1": 20, "config2": 100, "config3": 5}


def same_trees(gpu_trees: list[dict], o) -> bool:
    """Field-by-field equality of the library's first trees and all of the
    oracle's (structure, features, default directions exact; fp32 fields
    bit-exact)."""
    if len(gpu_trees) < o.num_trees() or o.num_trees() == 0:
        return False
    gpu_trees = gpu_trees[:o.num_trees()]
    for i, t in enumerate(gpu_trees):
        ot = o.tree(i)
        for f in ("left_children", "right_children", "split_indices", "default_left"):
            if not np.array_equal(np.array(t[f], np.int64), ot[f].astype(np.int64)):
                return False
        for f in ("split_conditions", "base_weights", "loss_changes", "sum_hessian"):
            if not np.array_equal(np.array(t[f], np.float32).view(np.uint32), ot[f].view(np.uint32)):
                return False
    return True


def config_runs(torch, dp, device, peak_gbs: float, threads: int, cpu: bool) -> list[dict]:
    """Configs 1-3 at full size on one GPU: one whole training run (every
    round, from a new booster; the DMatrix built before) timed with CUDA events
    after an identical untimed run; inputs resident in HBM.  Beside each, the
    CPU oracle on the same data (configs 1-2 in full, config 3 for its first
    five rounds) and whether its trees equal the GPU run's first trees."""
    sys.path.insert(0, str(ROOT / "oracle"))
    out = []
    for name, make, hp, rounds, K in CONFIGS:
        x, y = make(torch, device)
        R, F = x.shape
        params = {"tree_method": "hist", "max_bin": 256, "eta": 0.3, "lambda": 1.0, "min_child_weight": 1.0,
                  "device": f"cuda:{device.index or 0}"} | hp
        t0 = time.perf_counter()
        d = dp.DMatrix.from_torch(x, y)
        torch.cuda.synchronize()
        dmatrix_ms = 1e3 * (time.perf_counter() - t0)
        # the untimed run records every instrumented launch's events (where
        # a round's time goes); the timed run (identical trees) records none
        for timed in (False, True):
            b = dp.Booster(params, [d])
            b.set_profiling(not timed)
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            ev0.record()
            for i in range(rounds):
                b.update(d, i)
            ev1.record()
            torch.cuda.synchronize()
            if not timed:
                prof_all = b.profile()
                hist = prof_all.get("histograms", {"launches": 0, "ms": 0.0, "alg_bytes": 0.0})
                sections = {k: v["ms"] / rounds for k, v in prof_all.items()
                            if isinstance(v, dict) and "ms" in v and "launches" in v}
                b.free()
        ms = ev0.elapsed_time(ev1)
        trees = b.trees()
        b.free()
        d.free()
        line = {"config": name, "rows": R, "features": F, "max_depth": hp["max_depth"], "rounds": rounds,
                "trees_per_round": K, "objective": hp["objective"], "ms_total": ms,
                "ms_per_tree": ms / (rounds * K), "rows_trees_per_s": R * rounds * K / (ms / 1e3),
                "dmatrix_ms": dmatrix_ms,
                # per round, from the profiled run: the timed sections, and the
                # rest of the round (bookkeeping kernels, launch gaps, the host)
                "ms_per_round": {**{k: round(v, 4) for k, v in sorted(sections.items())},
                                 "rest": round(ms / rounds - sum(sections.values()), 4)},
                "histograms": {"launches": hist["launches"], "ms": hist["ms"],
                               "GBps": hist["alg_bytes"] / (hist["ms"] / 1e3) / 1e9 if hist["ms"] else 0.0,
                               "frac_hbm": (hist["alg_bytes"] / (hist["ms"] / 1e3) / 1e9 / peak_gbs)
                               if hist["ms"] else 0.0}}
        if name == "config3":
            line["l2_note"] = "47 MB of bins fit in the 126 MB L2: GB/s is HBM-equivalent"
        if cpu:
            import oracle
            xc, yc = x.cpu().numpy(), y.cpu().numpy()
            cr = CPU_ROUNDS[name]
            m = oracle.Model(xc, yc, hp["objective"], num_class=K, max_depth=hp["max_depth"], max_bin=256, eta=0.3,
                             rounds=0, threads=threads)
            t1 = time.perf_counter()
            m.train_more(cr)
            dt = time.perf_counter() - t1
            line["cpu_oracle"] = {"rounds": cr, "seconds": dt, "rows_trees_per_s": R * cr * K / dt,
                                  "cores": threads}
            line["trees_identical_to_oracle"] = same_trees(trees, m)
            line["trees_compared"] = m.num_trees()
            del m
        del x, y
        out.append(line)
        torch.cuda.empty_cache()
    return out


# --------------------------------------------------------------------------- CSV ingest
def csv_text(rows: int, cols: int, seed: int = SEED + 7) -> bytes:
    """Seeded CSV with a header and an integer class column: every feature is
    a fixed-width decimal  [-]ddd.dddd  (values of about N(0, 100)), built
    with numpy byte arithmetic so that hundreds of MB take seconds."""
    rng = np.random.default_rng(seed)
    v = np.clip(np.rint(rng.standard_normal((rows, cols)) * 1e6), -9999999, 9999999).astype(np.int64)
    neg = v < 0
    a = np.abs(v)
    width = 10  # sign or space, 3 digits, '.', 4 digits, ','
    cell = np.empty((rows, cols, width), np.uint8)
    cell[..., 0] = np.where(neg, ord("-"), ord(" "))
    for k, div in enumerate((10**6, 10**5, 10**4)):
        cell[..., 1 + k] = ord("0") + (a // div) % 10
    cell[..., 4] = ord(".")
    for k, div in enumerate((10**3, 10**2, 10, 1)):
        cell[..., 5 + k] = ord("0") + (a // div) % 10
    cell[..., 9] = ord(",")
    lab = rng.integers(0, 10, rows).astype(np.uint8)
    line = np.concatenate([cell.reshape(rows, cols * width), (ord("0") + lab)[:, None],
                           np.full((rows, 1), ord("\n"), np.uint8)], 1)
    head = (",".join(f"f{c}" for c in range(cols)) + ",label\n").encode()
    return head + line.tobytes()


def csv_bench(dp, peak_gbs: float, cpu: bool) -> dict:
    """GPU CSV decode (dp_csv_decode) of a 1M x 64 table (the config-2
    shape as text, 650 MB): device time (events, text already on the device)
    and end to end from host bytes; beside it the reference's own decoder
    (oracle/_ref/ref_csv, one host thread) on the first 20k rows."""
    rows, cols = 1_000_000, 64
    data = csv_text(rows, cols)
    for _ in range(2):
        dp.CsvTable(data, "label").free()
    ms_dev, ms_e2e = [], []
    for _ in range(3):
        t0 = time.perf_counter()
        t = dp.CsvTable(data, "label")
        ms_e2e.append(1e3 * (time.perf_counter() - t0))
        ms_dev.append(t.device_ms)
        assert (t.rows, t.features, t.classes) == (rows, cols, 10)
        t.free()
    dev, e2e = min(ms_dev), min(ms_e2e)
    out = {"rows": rows, "features": cols, "bytes": len(data), "device_ms": dev, "e2e_ms": e2e,
           "device_GBps": len(data) / (dev / 1e3) / 1e9, "e2e_GBps": len(data) / (e2e / 1e3) / 1e9,
           "device_frac_hbm_one_pass": len(data) / (dev / 1e3) / 1e9 / peak_gbs,
           "note": "device time excludes the host->device copy of the text and the allocation made once the "
                   "delimiters are counted; the text is read about four times (quote count, delimiter count and "
                   "write, field scan)"}
    ref = ROOT / "oracle" / "_ref" / "ref_csv"
    if cpu and ref.exists():
        import subprocess
        import tempfile
        sample_rows = 20_000
        cut = data.index(b"\n") + 1 + sample_rows * (cols * 10 + 2)
        with tempfile.TemporaryDirectory() as tmp:
            src = pathlib.Path(tmp) / "s.csv"
            src.write_bytes(data[:cut])
            subprocess.run([str(ref), str(src), "label", "auto", tmp, "3"], check=True, timeout=300)
            meta = json.loads((pathlib.Path(tmp) / "meta.json").read_text())
        out["cpu_reference"] = {"rows": sample_rows, "bytes": cut, "seconds": meta["seconds"],
                                "GBps": cut / meta["seconds"] / 1e9, "cores": 1,
                                "kind": "reference (decision_programs_csv::decode, built unmodified)"}
    return out


# --------------------------------------------------------------------------- histogram sweep (config 5)
def hist_sweep(torch, dp, device, peak_gbs: float, atomic_ceiling: float) -> list[dict]:
    R, F = 100_000_000, 32
    out = []
    g = torch.Generator(device=device)
    g.manual_seed(SEED + 5)
    gh = torch.stack([torch.randn(R, device=device, generator=g), torch.rand(R, device=device, generator=g)],
                     1).contiguous()
    for B in (16, 64, 256):
        bins = torch.randint(0, B, (R, F), dtype=torch.uint8, device=device, generator=g)
        for N in (1, 8, 64, 1024):
            node = torch.randint(0, N, (R,), device=device, generator=g)
            ridx = torch.argsort(node, stable=True).to(torch.int32)
            ghp = gh[ridx.long()].contiguous()
            dp.check(dp.lib().dp_quantize_gh(ghp.data_ptr(), R, 2.0 ** 15, 2.0 ** 16, None))
            counts = torch.bincount(node, minlength=N).cpu().numpy()
            del node
            edges = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
            sb, se = np.ascontiguousarray(edges[:-1]), np.ascontiguousarray(edges[1:])
            hist = torch.empty((N, F, 256, 2), dtype=torch.int64, device=device)
            plan = dp.ctypes_void_p()
            dp.check(dp.lib().dp_hist_prepare(bins.data_ptr(), F, F, B, 1, ghp.data_ptr(), ridx.data_ptr(), sb.ctypes.data,
                                              se.ctypes.data, N, 2.0 ** 15, 2.0 ** 16, hist.data_ptr(),
                                              dp.C.byref(plan)))
            stream = torch.cuda.current_stream()
            for _ in range(3):
                dp.check(dp.lib().dp_hist_run(plan, stream.cuda_stream))
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            reps = 5
            torch.cuda.synchronize()
            ev0.record()
            for _ in range(reps):
                dp.check(dp.lib().dp_hist_run(plan, stream.cuda_stream))
            ev1.record()
            torch.cuda.synchronize()
            ms = ev0.elapsed_time(ev1) / reps
            dp.check(dp.lib().dp_hist_free(plan))
            alg = R * (F + 12) + N * F * 256 * 16
            out.append({"bins": B, "nodes": N, "ms": round(ms, 4), "GB/s": round(alg / ms / 1e6, 1),
                        "frac_hbm": round(alg / ms / 1e6 / peak_gbs, 3),
                        "rows_features_per_s": R * F / (ms / 1e3),
                        "frac_atomic_ceiling": round(R * F / (ms / 1e3) / atomic_ceiling, 3) if atomic_ceiling else None})
            del ridx, ghp, hist
        del bins
    del gh
    torch.cuda.empty_cache()
    return out


def hist_sweep_sharded(torch, dp, device, comm, world: int, rank: int, peak_gbs: float, nccl_peak: dict,
                       max_over_ranks) -> list[dict]:
    """Config 5 with its 100M rows sharded over the ranks: every rank builds
    the partial histograms of its 100M/G rows, then the library's histogram
    exchange (a reduce-scatter of the int64 partials) leaves each rank the
    summed histograms of 1/G of the (node, feature) cells -- the feature
    groups (or node groups) it evaluates.  Time per case = the slowest rank's
    build + exchange (CUDA events on one stream, five launches after three
    warm-ups).  HBM fraction per GPU (its rows' algorithmic bytes plus its
    partial histograms); NVLink fraction against the NCCL reduce-scatter rate
    measured in this run."""
    R_total, F = 100_000_000, 32
    R = R_total // world
    out = []
    g = torch.Generator(device=device)
    g.manual_seed(SEED + 5 + 1000 * rank)
    gh = torch.stack([torch.randn(R, device=device, generator=g), torch.rand(R, device=device, generator=g)],
                     1).contiguous()
    stream = torch.cuda.current_stream()
    for B in (16, 64, 256):
        bins = torch.randint(0, B, (R, F), dtype=torch.uint8, device=device, generator=g)
        for N in (1, 8, 64, 1024):
            node = torch.randint(0, N, (R,), device=device, generator=g)
            ridx = torch.argsort(node, stable=True).to(torch.int32)
            ghp = gh[ridx.long()].contiguous()
            dp.check(dp.lib().dp_quantize_gh(ghp.data_ptr(), R, 2.0 ** 15, 2.0 ** 16, None))
            counts = torch.bincount(node, minlength=N).cpu().numpy()
            del node
            edges = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
            sb, se = np.ascontiguousarray(edges[:-1]), np.ascontiguousarray(edges[1:])
            hist = torch.empty((N, F, 256, 2), dtype=torch.int64, device=device)
            n_cells = hist.numel()
            assert n_cells % world == 0
            recv = torch.empty(n_cells // world, dtype=torch.int64, device=device)
            plan = dp.ctypes_void_p()
            dp.check(dp.lib().dp_hist_prepare(bins.data_ptr(), F, F, B, 1, ghp.data_ptr(), ridx.data_ptr(),
                                              sb.ctypes.data, se.ctypes.data, N, 2.0 ** 15, 2.0 ** 16,
                                              hist.data_ptr(), dp.C.byref(plan)))

            def step():
                dp.check(dp.lib().dp_hist_run(plan, stream.cuda_stream))
                comm.reduce_scatter_hist(hist.data_ptr(), recv.data_ptr(), n_cells // world, stream.cuda_stream)

            for _ in range(3):
                step()
            torch.cuda.synchronize()
            reps = 5
            e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            hist_ms = ex_ms = 0.0
            for _ in range(reps):
                e0.record()
                dp.check(dp.lib().dp_hist_run(plan, stream.cuda_stream))
                e1.record()
                comm.reduce_scatter_hist(hist.data_ptr(), recv.data_ptr(), n_cells // world, stream.cuda_stream)
                e2.record()
                torch.cuda.synchronize()
                hist_ms += e0.elapsed_time(e1) / reps
                ex_ms += e1.elapsed_time(e2) / reps
            dp.check(dp.lib().dp_hist_free(plan))
            ms = max_over_ranks(hist_ms + ex_ms)
            hist_ms, ex_ms = max_over_ranks(hist_ms), max_over_ranks(ex_ms)
            alg = R * (F + 12) + N * F * 256 * 16
            sent = n_cells * 8 * (world - 1) / world
            out.append({"bins": B, "nodes": N, "gpus": world, "ms": round(ms, 4), "hist_ms": round(hist_ms, 4),
                        "exchange_ms": round(ex_ms, 4),
                        "rows_features_per_s": R_total * F / (ms / 1e3),
                        "frac_hbm_per_gpu": round(alg / (hist_ms / 1e3) / 1e9 / peak_gbs, 3),
                        "nvlink_GBps": round(sent / (ex_ms / 1e3) / 1e9, 1),
                        "frac_nvlink": round(sent / (ex_ms / 1e3) / 1e9 / nccl_peak["GBps"], 3)})
            del ridx, ghp, hist, recv
        del bins
    del gh
    torch.cuda.empty_cache()
    return out


def hist_case(rows: int, nodes: int, nbins: int, features: int = 32) -> None:
    """One config-5 histogram case: random bins, seeded uniform row->node
    assignment, node-grouped row lists, quantised (g, h); three launches."""
    import ctypes
    import torch
    import dp_gbdt as dp
    g = torch.Generator(device="cuda")
    g.manual_seed(SEED + 5)
    bins = torch.randint(0, nbins, (rows, features), dtype=torch.uint8, device="cuda", generator=g)
    gh = torch.stack([torch.randn(rows, device="cuda", generator=g), torch.rand(rows, device="cuda", generator=g)],
                     1).contiguous()
    node = torch.randint(0, nodes, (rows,), device="cuda", generator=g)
    ridx = torch.argsort(node, stable=True).to(torch.int32)
    ghp = gh[ridx.long()].contiguous()
    dp.check(dp.lib().dp_quantize_gh(ghp.data_ptr(), rows, 2.0 ** 15, 2.0 ** 16, None))
    counts = torch.bincount(node, minlength=nodes).cpu().numpy()
    edges = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
    sb, se = np.ascontiguousarray(edges[:-1]), np.ascontiguousarray(edges[1:])
    hist = torch.empty((nodes, features, 256, 2), dtype=torch.int64, device="cuda")
    plan = ctypes.c_void_p()
    dp.check(dp.lib().dp_hist_prepare(bins.data_ptr(), features, features, nbins, 1, ghp.data_ptr(), ridx.data_ptr(),
                                      sb.ctypes.data, se.ctypes.data, nodes, 2.0 ** 15, 2.0 ** 16, hist.data_ptr(),
                                      ctypes.byref(plan)))
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(3):
        dp.check(dp.lib().dp_hist_run(plan, stream))
    torch.cuda.synchronize()
    dp.check(dp.lib().dp_hist_free(plan))
    print(json.dumps({"hist_case": [rows, nodes, nbins], "ok": True}))


# --------------------------------------------------------------------------- main GPU arm
def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="skip the config 1-3 runs")
    ap.add_argument("--no-csv", action="store_true", help="skip the CSV ingest measurement")
    ap.add_argument("--rows", type=int, default=ROWS,
                    help="total rows (default: config 4's 10M; smaller for profiler captures)")
    ap.add_argument("--hist-case", default=None,
                    help="ROWS,NODES,BINS: only run the config-5 histogram on one small case (3 launches), "
                         "for profilers")
    args = ap.parse_args()
    if args.impl == "reference":
        reference_arm(args)
        return
    if args.hist_case:
        hist_case(*(int(v) for v in args.hist_case.split(",")))
        return
    assert args.warmup >= 3, "at least 3 warm-up rounds"

    import torch
    import torch.distributed as dist

    import dp_gbdt as dp
    import ctypes
    dp.C = ctypes
    dp.ctypes_void_p = ctypes.c_void_p

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE={world}"
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=device)
    peaks = measured_peaks()
    peak_gbs = float(peaks["hbm_gbs"])

    assert args.rows % CHUNK == 0 and args.rows // CHUNK >= world, f"--rows must be a multiple of {CHUNK}"
    x, y = shard(torch, rank, world, device, args.rows)
    rows_local = x.shape[0]
    comm = None
    if world > 1:
        uid = torch.zeros(128, dtype=torch.uint8, device=device)
        if rank == 0:
            uid.copy_(torch.frombuffer(bytearray(dp.Comm.unique_id()), dtype=torch.uint8))
        dist.broadcast(uid, 0)
        comm = dp.Comm(bytes(uid.cpu().numpy().tobytes()), world, rank, local)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- the NVLink denominator: NCCL's reduce-scatter rate between these GPUs
    nccl_peak = measure_reduce_scatter(torch, dist, device, world, max_over_ranks) if world > 1 else None

    # ---- the histogram kernel's shared-atomic ceiling on this GPU (its bound)
    ceiling = dp.C.c_double(0.0)
    dp.check(dp.lib().dp_probe_hist_atomics(20000, dp.C.byref(ceiling), None))
    torch.cuda.synchronize()

    # ---- device-resident timing
    d = dp.DMatrix.from_torch(x, y)
    b = dp.Booster(PARAMS | {"device": f"cuda:{local}"}, [d])
    if comm is not None:
        b.set_comm(comm)
    # timing events around the histogram launches only (the least
    # instrumentation of the timed rounds), on from the start so that the
    # warm-up rounds capture the round graph with them; enabling again resets
    # the counters
    b.set_profiling(True, histograms_only=True)
    for i in range(args.warmup):
        b.update(d, i)
    b.set_profiling(True, histograms_only=True)
    clocks = ClockSampler(torch, local)
    clocks.start()
    barrier()
    launches0 = dp.launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for i in range(args.steps):
        b.update(d, args.warmup + i)
    ev1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    launches = dp.launch_count() - launches0
    ms_local = ev0.elapsed_time(ev1)
    barrier()
    ms = max_over_ranks(ms_local)
    hist = b.profile().get("histograms", {"launches": 0, "ms": 0.0, "alg_bytes": 0.0})
    # the per-kernel breakdown comes from a few more rounds with every launch
    # timed, after the timed region
    b.set_profiling(True)
    breakdown_rounds = 3
    for i in range(breakdown_rounds):
        b.update(d, args.warmup + args.steps + i)
    torch.cuda.synchronize()
    prof = {k: {**v, "launches_per_round": v["launches"] / breakdown_rounds, "ms_per_round": v["ms"] / breakdown_rounds}
            for k, v in b.profile().items() if isinstance(v, dict) and "ms" in v}
    # the rest of a timed round: bookkeeping kernels (decisions, task lists,
    # children, round start and read-back) and launch gaps
    prof["rest"] = {"ms_per_round": ms / args.steps - sum(v["ms_per_round"] for v in prof.values())}
    host_ms = b.profile().get("host_ms")
    levels = per_level(b.profile().get("log", []))
    value = args.rows * args.steps / (ms / 1e3)
    # NVLink: bytes this rank sends in the histogram reduce-scatter ((G-1)/G of
    # its partial histograms) over the exchange's event time, against the
    # reduce-scatter rate NCCL reaches between these GPUs at 1 GiB (measured
    # above, in this run)
    nvlink = None
    if world > 1 and "exchange_hist" in prof:
        ex = prof["exchange_hist"]
        sent = ex["alg_bytes"] * (world - 1) / world
        peak = nccl_peak["GBps"]
        nvlink = {"collective": "reduce-scatter of histogram partials + all-gather of split candidates",
                  "bytes_per_round_per_rank": sent / breakdown_rounds,
                  "achieved_GBps": sent / (ex["ms"] / 1e3) / 1e9 if ex["ms"] else 0.0,
                  "peak_GBps": peak, "peak_source": nccl_peak["how"],
                  "frac": (sent / (ex["ms"] / 1e3) / 1e9 / peak) if ex["ms"] and peak else 0.0,
                  "note": "exchange time includes waiting for the slowest rank's histogram"}
    hist_pairs_per_s = hist.get("units", 0.0) / (hist["ms"] / 1e3) if hist["ms"] else 0.0
    # the library's choice: 64-feature tasks on one GPU above 64 features
    # (DP_HIST_WIDE overrides), 32-feature tasks otherwise
    wide_env = os.environ.get("DP_HIST_WIDE", "")
    hist_kernel = "k_hist_wide" if (wide_env == "1" or (wide_env != "0" and world == 1 and FEATURES > 64)) \
        else "k_hist"
    atomic_roofline = {"kernel": hist_kernel, "unit": "(row, feature) pairs/s", "achieved": hist_pairs_per_s,
                       "ceiling": ceiling.value, "frac": hist_pairs_per_s / ceiling.value if ceiling.value else 0.0,
                       "ceiling_source": "dp_probe_hist_atomics: the kernel's shared-memory update loop alone "
                                         "(two 32-bit atomics per pair, one 1024-thread block per SM), "
                                         "measured in this run"}
    hist_ms_per_launch = hist["ms"] / max(1, hist["launches"])
    achieved = hist["alg_bytes"] / max(1, hist["launches"]) / (hist_ms_per_launch / 1e3) / 1e9 if hist["ms"] else 0.0
    # DRAM bytes per histogram launch of this workload, from the committed ncu
    # summary (one-pass capture of one full round at full size)
    traffic = None
    tfile = ROOT / "profiles" / "k_hist_config4_traffic.md"
    if tfile.exists() and args.rows == ROWS and world == 1:
        m = re.search(r"^bytes_per_launch_config4:\s*(\d+)", tfile.read_text(), re.M)
        traffic = int(m.group(1)) if m else None
    model_bytes = len(b.save_raw())
    # the first trees of this run, compared with the CPU oracle's below
    first_trees = b.trees()[:C4_PARITY_TREES] if (world == 1 and args.rows == ROWS and not args.no_cpu) else None
    b.free()
    d.free()

    # ---- end to end through the C-ABI with host buffers
    e2e = None
    if not args.no_e2e:
        e2e = end_to_end(torch, dp, x, y, args, local, comm, barrier, max_over_ranks, world)
    del x, y
    torch.cuda.empty_cache()

    sweep = None
    cpu = None
    configs = None
    csv = None
    if rank == 0 and world == 1:
        if not args.no_csv:
            csv = csv_bench(dp, peak_gbs, not args.no_cpu)
        if not args.no_configs:
            configs = config_runs(torch, dp, device, peak_gbs, len(os.sched_getaffinity(0)), not args.no_cpu)
        if not args.no_sweep:
            sweep = hist_sweep(torch, dp, device, peak_gbs, ceiling.value)
        if not args.no_cpu and first_trees is not None:
            cpu = config4_cpu_leg(torch, first_trees)
    if world > 1 and not args.no_sweep:
        sweep = hist_sweep_sharded(torch, dp, device, comm, world, rank, peak_gbs, nccl_peak, max_over_ranks)
    if comm is not None:
        comm.free()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": "boosting rows*trees/s (config 4 step, 1 tree)", "value": value, "unit": "rows*trees/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u8 bins / int64 sums",
        "data": "synthetic (seeded), inputs larger than L2",
        "config": workload_config(args.rows),
        "parallelism": f"rows sharded over {world} GPU(s)",
        "e2e": e2e,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak_gbs, "unit": "GB/s",
                     "frac": achieved / peak_gbs, "traffic": traffic, "kernel": hist_kernel,
                     "peak_source": "measured" if not peaks.get("fallback") else "fallback",
                     "launches": hist["launches"], "ms_per_launch": hist_ms_per_launch},
        "rows_features_per_s": value * FEATURES,
        "atomic_roofline": atomic_roofline,
        "gpu_launches": launches,
        "clocks": clk,
        "kernel_profile": prof,
        "nvlink": nvlink,
        "levels_last_round": levels,
        "host_ms": host_ms,
        "model_bytes": model_bytes,
    }
    if cpu is not None:
        line["trees_identical_to_oracle"] = cpu.pop("trees_identical_to_oracle")
        line["trees_compared"] = cpu.pop("trees_compared")
        third = cpu.pop("third_party", None)
        line["cpu_baseline"] = cpu
        if third is not None:
            line["cpu_third_party"] = third
    if sweep is not None:
        line["hist_sweep"] = sweep
    if configs is not None:
        line["configs"] = configs
    if csv is not None:
        line["csv_ingest"] = csv
    print(json.dumps(line), flush=True)


def measure_reduce_scatter(torch, dist, device, world: int, max_over_ranks) -> dict:
    """Bytes each rank sends per second in an NCCL reduce-scatter of 1 GiB of
    int64 per rank ((G-1)/G of the input crosses NVLink), the slowest rank's
    time over ten back-to-back calls after three warm-up calls."""
    n = (1 << 27) // world * world
    inp = torch.ones(n, dtype=torch.int64, device=device)
    out = torch.empty(n // world, dtype=torch.int64, device=device)
    for _ in range(3):
        dist.reduce_scatter_tensor(out, inp)
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 10
    e0.record()
    for _ in range(reps):
        dist.reduce_scatter_tensor(out, inp)
    e1.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / reps)
    sent = n * 8 * (world - 1) / world
    del inp, out
    torch.cuda.empty_cache()
    return {"GBps": sent / (ms / 1e3) / 1e9, "ms": ms,
            "how": "NCCL reduce-scatter of 1 GiB int64 per rank between these GPUs, measured in this run "
                   "(bytes sent per rank / time, slowest rank)"}


def per_level(log: list) -> list[dict]:
    """Per-depth device times (ms) of the last profiled round, from the
    profiler's launch log [name, ms, bytes] in launch order: a round starts at
    'gradients' and every 'histograms' entry starts a level."""
    starts = [i for i, e in enumerate(log) if e[0] == "gradients"]
    if not starts:
        return []
    levels: list[dict] = []
    for name, ms, _ in log[starts[-1]:]:
        if name == "histograms":
            levels.append({})
        if levels:
            levels[-1][name] = round(levels[-1].get(name, 0.0) + ms, 4)
    return levels


def end_to_end(torch, dp, x, y, args, local, comm, barrier, max_over_ranks, world) -> dict:
    """The metric through the C-ABI from pinned host buffers: the host matrix
    goes in through XGDMatrixCreateFromDense (upload overlapped with the first
    cut-counting pass), labels through XGDMatrixSetFloatInfo, then W+K rounds
    and the JSON model read back."""
    xh = torch.empty_like(x, device="cpu").pin_memory()
    yh = torch.empty_like(y, device="cpu").pin_memory()
    xh.copy_(x)
    yh.copy_(y)
    rounds_e2e = args.warmup + args.steps
    trials, dmatrix_ms = [], []
    for _ in range(3):  # whole-job trials; the median is reported
        barrier()
        e0, em, e1 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record()
        d2 = dp.DMatrix.from_host(xh, yh)
        b2 = dp.Booster(PARAMS | {"device": f"cuda:{local}"}, [d2])
        if comm is not None:
            b2.set_comm(comm)
        b2.update(d2, 0)  # builds the cuts and bins, then the first round
        em.record()
        for i in range(1, rounds_e2e):
            b2.update(d2, i)
        raw = b2.save_raw()
        e1.record()
        torch.cuda.synchronize()
        trials.append(max_over_ranks(e0.elapsed_time(e1)))
        dmatrix_ms.append(max_over_ranks(e0.elapsed_time(em)))
        b2.free()
        d2.free()
    e2e_ms = statistics.median(trials)
    return {"value": args.rows * rounds_e2e / (e2e_ms / 1e3), "unit": "rows*trees/s",
            "h2d_bytes_per_step": int(args.rows * (FEATURES + 1) * 4 / rounds_e2e),
            "d2h_bytes_per_step": int(len(raw) * world / rounds_e2e),
            "trials_ms": trials, "first_round_ms": statistics.median(dmatrix_ms),
            "note": f"pinned host fp32 inputs -> XGDMatrixCreateFromDense (upload + cuts + bins) -> "
                    f"{rounds_e2e} rounds -> JSON model; median of 3 whole-job trials; first_round_ms = "
                    f"upload, cuts, bins and the first round"}


if __name__ == "__main__":
    main()
