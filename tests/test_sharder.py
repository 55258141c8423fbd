"""Row-block sharder host logic: block bounds, and a world_size-2 gloo run on
CPU where each rank computes its rows with the CPU oracle, all-gathers the C
blocks and re-lays them out; the result must equal the unsharded oracle GEMM
bit for bit (every element is computed by the same code in the same order)."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import sharder


def test_row_blocks_cover_and_align():
    for m, world, align in ((4096, 1, 256), (32768, 8, 256), (8192, 3, 256), (520, 2, 64),
                            (1000, 4, 8), (256, 4, 256)):
        blocks = sharder.row_blocks(m, world, align)
        assert len(blocks) == world
        assert blocks[0].row0 == 0
        assert sum(b.rows for b in blocks) == m
        for a, b in zip(blocks, blocks[1:]):
            assert b.row0 == a.row0 + a.rows
        for b in blocks[:-1]:
            assert b.rows % align == 0
        assert max(b.rows for b in blocks) - min(b.rows for b in blocks if b.rows) < 2 * align
    blocks = sharder.row_blocks(32768, 8)
    assert all(b.rows == 4096 for b in blocks)
    with pytest.raises(ValueError):
        sharder.row_blocks(1024, 2, align=12)


def test_relayout_places_blocks():
    blocks = sharder.row_blocks(24, 3, align=8)
    n, pad = 5, 8
    g = torch.arange(3 * n * pad, dtype=torch.float32).reshape(3, n, pad)
    c = sharder.relayout(g.reshape(-1), blocks, n)
    for b in blocks:
        assert torch.equal(c[:, b.row0:b.row0 + b.rows], g[b.rank, :, :b.rows])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, m, n, k, layout, q):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    for p in (os.path.join(root, "best-matmul_b200"), os.path.join(root, "oracle")):
        sys.path.insert(0, p)
    import sharder as sh
    from oracle import Oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        orc = Oracle()
        blocks = sh.row_blocks(m, world, align=64)
        blk = blocks[rank]
        pad = sh.max_rows(blocks)
        # this rank's rows of A (row-major logical rows, any layout: the
        # generator depends on the logical index only) and all of B
        a_rows = orc.fill(blk.rows, k, k, 1, blk.row0, k, 4, 0, 0)
        b_full = orc.fill(n, k, k, 1, 0, k, 4, 0, 1)
        c_blk = orc.gemm_f32(k, "TN", a_rows, k, b_full, k, 0, blk.rows, 0, n)  # (n, rows)
        c_local = torch.zeros((n, pad), dtype=torch.float16)
        c_local[:, :blk.rows] = torch.from_numpy(c_blk.astype(np.float16))
        c_global = sh.gather_c(c_local, blocks, n)
        if rank == 0:
            a_all, b_all = orc.make_inputs(m, n, k, "TN", 4, seed=0)
            ref = orc.gemm_f32(k, "TN", a_all, k, b_all, k, 0, m, 0, n).astype(np.float16)
            q.put(bool(np.array_equal(c_global.numpy(), ref)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("m", [512, 448])
def test_gloo_two_ranks_match_unsharded(m):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, m, 96, 80, "TN", q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=5) is True
