"""Sharded GEMM on GPU: every rank's row block (here: each rank of a P-way
split run in turn on one GPU) equals the corresponding rows of the global
GEMM, checked on sampled entries against the FP64 oracle; and the BASELINE
configs[4] size (32768^3 NT) on one GPU, sampled."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-2, 2e-3


def _sampled_check(orc, sg, n_samples=256, seed=0):
    """Compare sampled entries of this rank's C block with FP64 references
    computed from the rank's own A rows and B (copied back to the host)."""
    m_rows, n, k = sg.block.rows, sg.n, sg.k
    rng = np.random.default_rng(seed)
    rows = rng.integers(0, m_rows, n_samples)
    cols = rng.integers(0, n, n_samples)
    a = sg.a.cpu().numpy().view(np.uint16).reshape(-1)
    b = sg.b.cpu().numpy().view(np.uint16).reshape(-1)
    lda = sg.pad if sg.layout == "NT" else k
    ldb = n if sg.layout == "NT" else k
    ref = orc.entries_f64(k, sg.layout, a, lda, b, ldb, rows, cols)
    c = sg.c.cpu().numpy().view(np.uint16)
    got = np.ascontiguousarray(c[cols, rows])
    return orc.check(got, ref, k, RTOL, ATOL)


@pytest.mark.parametrize("layout", ["NT", "TN"])
def test_each_rank_block_matches_global_rows(orc, cuda, layout):
    import sharder
    m, n, k = 2048, 1024, 512
    world = 4
    # generator consistency: rank blocks are rows of the same global matrix
    full_a, _ = orc.make_inputs(m, n, k, layout, 4, seed=0)
    full_rows = full_a.reshape(k, m).T if layout == "NT" else full_a.reshape(m, k)
    for rank in range(world):
        sg = sharder.ShardedGemm(m, n, k, layout, rank, world)
        sg.launch()
        assert sg.gemm.status() == (0, 0)
        a = sg.a.cpu().numpy().view(np.uint16)
        blk = a[:, :sg.block.rows].T if layout == "NT" else a[:sg.block.rows]
        assert np.array_equal(blk, full_rows[sg.block.row0:sg.block.row0 + sg.block.rows])
        bad, merr, _ = _sampled_check(orc, sg, seed=rank)
        assert bad == 0, f"rank {rank}: {bad} bad samples, max err {merr}"
        sg.close()


def test_baseline_sharded_config_single_gpu(orc, cuda):
    """configs[4] at P = 1: 32768^3 NT, uniform[-1,1]."""
    import sharder
    sg = sharder.ShardedGemm(32768, 32768, 32768, "NT", 0, 1)
    sg.launch()
    assert sg.gemm.status() == (0, 0)
    bad, merr, _ = _sampled_check(orc, sg, n_samples=192)
    assert bad == 0, f"{bad} bad samples, max err {merr}"
    sg.close()
