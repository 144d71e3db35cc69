"""Failure detection of the multi-GPU path, host side: the polling wait
(decision-programs_b200/csrc/watchdog.h) that the training engine uses instead
of a blocking stream synchronisation while NCCL collectives are in flight.  A
peer that stops or fails must end in an abort of the communicator and an
error, never in a wait without end.  Runs on the CPU against fake completion,
error and abort functions (the GPU case is in test_gpu_multi.py)."""
import json
import pathlib
import shutil
import subprocess

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def cases(tmp_path_factory):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not found")
    exe = tmp_path_factory.mktemp("watchdog") / "watchdog_check"
    subprocess.run([gxx, "-std=c++17", "-O1", "-I", str(ROOT / "decision-programs_b200" / "csrc"),
                    str(ROOT / "tests" / "watchdog_check.cpp"), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True, timeout=60).stdout
    return {c["case"]: c for c in map(json.loads, out.splitlines())}


def test_completion_returns_without_abort(cases):
    c = cases["completes"]
    assert c["reason"] == "" and c["aborts"] == 0 and c["polls"] == 5


def test_asynchronous_error_aborts_once(cases):
    c = cases["error"]
    assert c["aborts"] == 1 and c["polls"] == 3
    assert "asynchronous communicator error: remote process exited" in c["reason"]


def test_deadline_aborts_once(cases):
    c = cases["timeout"]
    assert c["aborts"] == 1
    assert c["reason"].startswith("no completion within 20 ms")
    assert 20.0 <= c["ms"] < 2000.0


def test_no_deadline_waits_for_completion(cases):
    c = cases["no_deadline"]
    assert c["reason"] == "" and c["aborts"] == 0 and c["ms"] >= 50.0


def test_completion_is_checked_before_errors(cases):
    c = cases["done_before_error"]
    assert c["reason"] == "" and c["aborts"] == 0
