"""The data-parallel watchdog's logic without a GPU: veda_b200/csrc/host/watchdog.hpp compiled
with fake stream / communicator polls and a fake clock (tests/native/watchdog_check.cpp). A peer
that fails is seen either as an asynchronous communicator error or as no progress within the
timeout; either way the communicator is aborted exactly once and the wait ends with that
outcome instead of hanging."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def outcomes(tmp_path_factory):
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("no C++ compiler")
    exe = tmp_path_factory.mktemp("wd") / "watchdog_check"
    subprocess.run([cxx, "-std=c++20", "-O1", "-I", str(ROOT / "veda_b200" / "csrc" / "host"),
                    str(ROOT / "tests" / "native" / "watchdog_check.cpp"), "-o", str(exe)],
                   check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    return {line.split()[0]: line.split()[1:] for line in out.strip().splitlines()}


def test_completion_is_reported_without_abort(outcomes):
    assert outcomes["completes"] == ["done", "polls=5", "aborts=0"]


def test_communicator_error_aborts_once(outcomes):
    assert outcomes["peer_error"] == ["comm_error", "polls=3", "aborts=1"]


def test_no_progress_times_out_and_aborts_once(outcomes):
    kind, polls, aborts = outcomes["no_progress"]
    assert kind == "timeout" and aborts == "aborts=1"
    assert int(polls.split("=")[1]) == 10   # 2 s at 0.25 s per poll, then the timeout


def test_stream_error_is_reported_without_abort(outcomes):
    assert outcomes["stream_fault"] == ["stream_error", "polls=2", "aborts=0"]
