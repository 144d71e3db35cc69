"""Worker of tests/test_sharded_oracle.py: one gloo rank training its shard
of the rows with the sharded oracle (spawned by torch.multiprocessing)."""
import os
import pathlib
import sys

ROOT = pathlib.Path(__file__).resolve().parents[1]


def run(rank: int, world: int, port: int, x, y, kw: dict, out: dict) -> None:
    sys.path.insert(0, str(ROOT / "oracle"))
    import numpy as np
    import torch
    import torch.distributed as dist
    import oracle

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        def allreduce(buf, op):
            t = torch.from_numpy(buf)  # shares memory with the oracle's buffer
            dist.all_reduce(t, op=dist.ReduceOp.SUM if op == 0 else dist.ReduceOp.MAX)

        lo, hi = rank * len(y) // world, (rank + 1) * len(y) // world
        m = oracle.Model.sharded(x[lo:hi], y[lo:hi], allreduce, **kw)
        out[rank] = {"trees": [m.tree(i) for i in range(m.num_trees())], "margins": m.margins(),
                     "cuts": m.cuts()}
    finally:
        dist.destroy_process_group()
