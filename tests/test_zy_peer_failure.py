"""Failure detection of row-sharded training on 2 GPUs (one process per GPU,
NCCL communicator): a rank that stops must end the others' round in an error
from the communicator's watchdog, not in a wait without end.  The failure is
made on the host (a rank leaves between rounds); NVLS stays off.  Collected
after the other GPU tests.  Skipped on a box with fewer than two GPUs."""
import json
import os
import pathlib
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
ROOT = pathlib.Path(__file__).resolve().parents[1]


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs at least two GPUs")
def test_a_peer_that_stops_ends_in_an_error(tmp_path):
    """Failure detection: rank 1 leaves after the first round (between rounds,
    nothing in flight); rank 0's second round must end within seconds in an
    error naming the aborted communicator, not wait for good.  NVLS stays off."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "180", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={free_port()}",
           str(ROOT / "tests" / "_multi_gpu_worker.py"), "peer_stops", str(tmp_path), "2"]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.loads((tmp_path / "rank0_failure.json").read_text())
    assert "NCCL communicator of rank 0 aborted" in res["error"], res
    assert res["seconds"] < 60.0, res
