"""The bounded host wait of a tensor-parallel engine step (alb_wait.h), on the
CPU with fake probes: a finished stream returns at once, a stream or NCCL
error is reported, and a peer that never answers ends in a timeout near the
limit (after which the engine aborts its communicator).  No GPU."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def results(tmp_path_factory):
    cxx = shutil.which("g++")
    if not cxx:
        pytest.skip("no g++")
    exe = str(tmp_path_factory.mktemp("wait") / "wait_driver")
    subprocess.run([cxx, "-O2", "-std=c++17", "-pthread", "-I" + os.path.join(ROOT, "arclight_b200", "csrc"),
                    os.path.join(ROOT, "tests", "wait_driver.cpp"), "-o", exe], check=True)
    out = subprocess.run([exe], capture_output=True, text=True, check=True, timeout=60).stdout
    return {f[0]: (int(f[1]), int(f[2]), float(f[3])) for f in (l.split() for l in out.splitlines())}


def test_finished_stream(results):
    assert results["done"][:2] == (0, 100)
    assert results["done_first"][:2] == (0, 1)


def test_errors_are_reported(results):
    assert results["stream_error"][:2] == (1, 10)
    assert results["comm_error"][:2] == (2, 50)


def test_silent_peer_times_out_near_the_limit(results):
    code, polls, ms = results["timeout"]
    assert code == 3 and polls > 1
    assert 50.0 <= ms < 1000.0
