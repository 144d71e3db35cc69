"""Worker of tests/test_gpu_multi.py, launched by torch.distributed.run: one
process per GPU trains its shard of the rows through libdp_gbdt with an NCCL
communicator and writes its model and margins to OUT_DIR/rank{r}.*

Case "peer_stops": after the first round every rank but 0 leaves the job
(between rounds, with nothing of its own in flight); rank 0 runs the second
round with a 3-second communicator deadline and writes what happened to
OUT_DIR/rank0_failure.json."""
import datetime
import json
import os
import pathlib
import sys
import time

ROOT = pathlib.Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "decision-programs_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import dp_gbdt as dp  # noqa: E402


def data(case: str):
    rng = np.random.default_rng(11)
    R, F = 40_003, 24
    x = rng.standard_normal((R, F)).astype(np.float32)
    if case == "logistic_nan":
        x[rng.random((R, F)) < 0.1] = np.nan
        y = (np.nan_to_num(x[:, 0]) + 0.5 * np.nan_to_num(x[:, 1]) > 0).astype(np.float32)
        return x, y, {"objective": "binary:logistic", "max_depth": 6}
    if case == "wide":
        # 100 features: two 64-feature histogram tiles, each spanning both
        # ranks' feature groups
        x = rng.standard_normal((R, 100)).astype(np.float32)
        y = (x[:, 3] * x[:, 70] + np.sin(x[:, 99]) + 0.1 * rng.standard_normal(R)).astype(np.float32)
        return x, y, {"objective": "reg:squarederror", "max_depth": 6}
    if case == "softprob":
        y = np.argmax(x[:, :4] + 0.3 * rng.standard_normal((R, 4)), 1).astype(np.float32)
        return x, y, {"objective": "multi:softprob", "num_class": 4, "max_depth": 5}
    y = (x[:, 0] * x[:, 1] + np.sin(x[:, 2]) + 0.1 * rng.standard_normal(R)).astype(np.float32)
    if case == "deep_exact_host":
        return x, y, {"objective": "reg:squarederror", "max_depth": 11, "min_child_weight": 0.0}
    if case == "sampled":
        return x, y, {"objective": "reg:squarederror", "max_depth": 6, "subsample": 0.7, "colsample_bytree": 0.8,
                      "colsample_bynode": 0.5, "seed": 77}
    return x, y, {"objective": "reg:squarederror", "max_depth": 8}


def peer_stops(params: dict, d, comm, rank: int, out_dir: pathlib.Path) -> None:
    b = dp.Booster(params, [d])
    b.set_comm(comm)
    b.update(d, 0)
    torch.cuda.synchronize()
    comm.set_timeout(3000)  # the first round keeps the default, which covers start-up skew
    dist.barrier()  # every rank has finished the first round
    if rank != 0:
        os._exit(0)  # leaves without a word to the others; none of its work is in flight
    t0 = time.monotonic()
    try:
        b.update(d, 1)
        error = ""
    except dp.DPError as e:
        error = str(e)
    (out_dir / "rank0_failure.json").write_text(json.dumps({"error": error, "seconds": time.monotonic() - t0}))
    sys.stdout.flush()
    os._exit(0)  # the process group and the communicator cannot be closed with a peer gone


def main() -> None:
    case, out_dir, rounds = sys.argv[1], pathlib.Path(sys.argv[2]), int(sys.argv[3])
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    try:
        uid = torch.zeros(128, dtype=torch.uint8)
        if rank == 0:
            uid.copy_(torch.frombuffer(bytearray(dp.Comm.unique_id()), dtype=torch.uint8))
        dist.broadcast(uid, 0)
        comm = dp.Comm(bytes(uid.numpy().tobytes()), world, rank, local)
        x, y, params = data(case)
        lo, hi = rank * len(y) // world, (rank + 1) * len(y) // world
        if case.endswith("_host"):
            d = dp.DMatrix.from_host(np.ascontiguousarray(x[lo:hi]), np.ascontiguousarray(y[lo:hi]))
        else:
            d = dp.DMatrix.from_torch(torch.from_numpy(x[lo:hi]).cuda(), torch.from_numpy(y[lo:hi]).cuda())
        if case == "peer_stops":
            peer_stops(params | {"device": f"cuda:{local}"}, d, comm, rank, out_dir)
        b = dp.train(params | {"device": f"cuda:{local}"}, d, rounds, comm=comm)
        K = params.get("num_class", 1)
        (out_dir / f"rank{rank}.json").write_bytes(b.save_raw())
        np.save(out_dir / f"rank{rank}_margins.npy", b.margins(hi - lo, K))
        b.free()
        d.free()
        comm.free()
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
