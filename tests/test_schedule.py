"""CPU check of the persistent-grid schedule (best-matmul_b200/csrc/schedule.cuh).

tests/native/schedule_check.cpp compiles the kernel's own planner and work
iterator as plain C++ and runs them for every cluster of a grid over a sweep
of tile counts, part counts and cluster counts: every column part of every
tile is computed exactly once, whole tiles fill complete waves before any
split run, and no cluster gets more than the planned run of parts.
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


def _plan(checker, tiles, parts, clusters, split=1):
    out = subprocess.run([checker, str(tiles), str(parts), str(clusters), str(split)],
                         capture_output=True, text=True)
    assert out.returncode == 0, out.stdout
    m = re.search(r"plan dp_tiles=(\d+) tail_parts=(\d+) tail_clusters=(\d+) grid=(\d+)", out.stdout)
    return tuple(int(x) for x in m.groups())


def test_schedule_sweep(checker):
    out = subprocess.run([checker], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stdout[-3000:]
    assert re.search(r"\d+ cases, 0 failures", out.stdout)


def test_bench_shape_stays_whole(checker):
    """4096^3 with 256x512 pair tiles: 128 tiles on 74 resident pairs leave
    54 for the last wave, more than half the pairs: halves would still take a
    whole tile-time, so nothing is split."""
    assert _plan(checker, 128, 2, 74) == (128, 0, 0, 74)
    assert _plan(checker, 512, 2, 74) == (512, 0, 0, 74)   # 8192^3
    assert _plan(checker, 148, 2, 74) == (148, 0, 0, 74)
    assert _plan(checker, 256, 2, 74, split=0) == (256, 0, 0, 74)
    assert _plan(checker, 256, 1, 74) == (256, 0, 0, 74)


def test_small_remainder_is_halved(checker):
    """4096 x 8192: 256 tiles = 3 full waves + 34; the 68 halves go to 68
    pairs, so the last wave takes half a tile-time."""
    assert _plan(checker, 256, 2, 74) == (222, 68, 68, 74)


def test_fewer_tiles_than_clusters(checker):
    """2048^3 pair tiles: 32 tiles, their 64 halves over 64 pairs."""
    assert _plan(checker, 32, 2, 74) == (0, 64, 64, 64)
