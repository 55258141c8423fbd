"""CPU check of the persistent-grid schedule (best-matmul_b200/csrc/schedule.cuh).

tests/native/schedule_check.cpp compiles the kernel's own planner and work
iterator as plain C++ and runs them for every cluster of a grid over a sweep
of tile counts, quarter counts and cluster counts: every column quarter of
every tile is computed exactly once, whole tiles fill complete waves before
any split run, and no cluster gets more than the planned run of quarters.
"""
from __future__ import annotations

import os
import re
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "native", "schedule_check.cpp")
INC = os.path.join(ROOT, "best-matmul_b200", "csrc")


@pytest.fixture(scope="module")
def checker(tmp_path_factory):
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        pytest.fail("no C++ compiler")
    exe = str(tmp_path_factory.mktemp("sched") / "schedule_check")
    subprocess.run([cxx, "-O2", "-std=c++17", "-Wall", "-Werror", f"-I{INC}", SRC, "-o", exe],
                   check=True)
    return exe


def _plan(checker, tiles, quarters, clusters, split=1):
    out = subprocess.run([checker, str(tiles), str(quarters), str(clusters), str(split)],
                         capture_output=True, text=True)
    assert out.returncode == 0, out.stdout
    m = re.search(r"plan dp_tiles=(\d+) tail_quarters=(\d+) tail_clusters=(\d+) grid=(\d+)", out.stdout)
    return tuple(int(x) for x in m.groups())


def test_schedule_sweep(checker):
    out = subprocess.run([checker], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stdout[-3000:]
    assert re.search(r"\d+ cases, 0 failures", out.stdout)


def test_bench_shape(checker):
    """4096^3 with 256x512 pair tiles: 128 tiles on 74 resident pairs. One
    whole wave of 74 tiles; the other 54 tiles' 216 quarters go to 72 pairs
    in runs of 3, so the last wave takes 3/4 of a tile-time."""
    assert _plan(checker, 128, 4, 74) == (74, 216, 72, 74)


def test_nearly_full_waves_stay_whole(checker):
    """8192^3: 512 tiles, remainder 68 of 74: runs would be 4 quarters."""
    assert _plan(checker, 512, 4, 74) == (512, 0, 0, 74)
    assert _plan(checker, 148, 4, 74) == (148, 0, 0, 74)
    assert _plan(checker, 128, 4, 74, split=0) == (128, 0, 0, 74)
    assert _plan(checker, 128, 1, 74) == (128, 0, 0, 74)


def test_fewer_tiles_than_clusters(checker):
    """2048^3 pair tiles: 32 tiles, 128 quarters in runs of 2 over 64 pairs."""
    assert _plan(checker, 32, 4, 74) == (0, 128, 64, 64)
