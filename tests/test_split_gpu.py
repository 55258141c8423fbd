"""GPU checks of the split schedule (leftover tiles computed as 256-column
halves, best-matmul_b200/csrc/schedule.cuh) through the C ABI.

A split launch computes every output element with one MMA chain over all of
K in the same order as a whole-tile launch, so the two must agree bit for
bit; integer inputs (reference modes 1..3) must also match the exact result
bit for bit, and uniform inputs the CPU oracle within the tolerance
    |c - ref| <= 1e-2 * |ref| + 2e-3 * sqrt(K / 4096).
"""
from __future__ import annotations

import numpy as np
import pytest

from test_gemm_gpu import ATOL, RTOL, _bits, _describe_mismatch, _lds, _to_dev

pytestmark = pytest.mark.gpu

V5 = 5  # BM_VARIANT_2CTA_256x512, the variant whose leftover tiles split


def _run(bm, a, b, c, layout, mode, variant=V5, launches=1):
    with bm.Gemm.from_tensors(a, b, c, layout, variant=variant) as g:
        g.set_split(mode)
        sched = g.schedule()
        for _ in range(launches):
            g.launch()
        rc, bits = g.status()
    assert rc == bm.BM_OK, f"kernel status {rc}, device bits {bits:#x}"
    return sched


# (m, n, k): tile counts with a last wave of at most half the pairs (or fewer
# tiles than pairs), ragged N blocks and ragged M / N / K edges.
SHAPES = [
    (512, 1024, 384),    # 4 tiles: 8 halves
    (2048, 1280, 256),   # 24 tiles, last N block half empty: 48 halves
    (1792, 2048, 192),   # 28 tiles: 56 halves
    (1800, 1992, 136),   # ragged M, N and K: 32 tiles
    (4096, 8192, 320),   # 256 tiles: 3 whole waves, then 34 tiles as 68 halves
]


@pytest.mark.parametrize("layout", ["NT", "TN"])
@pytest.mark.parametrize("shape", SHAPES, ids=[f"{m}x{n}x{k}" for m, n, k in SHAPES])
def test_split_matches_whole_tiles_bitwise(bm, orc, cuda, layout, shape):
    torch = cuda
    m, n, k = shape
    if bm.check(m, n, k, layout) != bm.BM_OK:
        pytest.skip("leading dimension not a multiple of 8 for this layout")
    a, b, c = bm.alloc_operands(m, n, k, layout, mode=4, seed=11)
    c_whole = torch.full_like(c, float("nan"))
    c.fill_(float("nan"))
    s_none = _run(bm, a, b, c_whole, layout, bm.SPLIT_NONE)
    s_auto = _run(bm, a, b, c, layout, bm.SPLIT_AUTO, launches=2)
    assert s_none["split_parts"] == 0
    assert s_auto["split_parts"] > 0, s_auto
    got, want = _bits(c), _bits(c_whole)
    assert np.array_equal(got, want), _describe_mismatch(got, want, m, n, 256, 512)
    ea, eb = orc.make_inputs(m, n, k, layout, 4, seed=11)
    lda, ldb = _lds(m, n, k, layout)
    ref = orc.gemm_f32(k, layout, ea, lda, eb, ldb, 0, m, 0, n).astype(np.float64)
    bad, merr, worst = orc.check(got, ref, k, RTOL, ATOL)
    assert bad == 0, f"{bad} outside tolerance, max err {merr}, worst {worst}"


@pytest.mark.parametrize("layout", ["NT", "TN"])
def test_split_exact_integers(bm, orc, cuda, layout):
    """Reference input modes 1..3, NaN-prefilled C, two launches, every
    element bit for bit against the FP16 rounding of the exact result."""
    torch = cuda
    m, n, k = 1792, 2048, 320
    lda, ldb = _lds(m, n, k, layout)
    for mode in (1, 2, 3):
        ea, eb = orc.make_inputs(m, n, k, layout, mode)
        a, b, c = _to_dev(torch, ea, eb, m, n, k, layout)
        sched = _run(bm, a, b, c, layout, bm.SPLIT_AUTO, launches=2)
        assert sched["split_parts"] > 0
        want = orc.gemm_f32(k, layout, ea, lda, eb, ldb, 0, m, 0, n).astype(np.float16).view(np.uint16)
        got = _bits(c)
        assert np.array_equal(got, want), f"mode {mode}: " + _describe_mismatch(got, want, m, n, 256, 512)


@pytest.mark.parametrize("layout", ["NT", "TN"])
def test_bench_shape_schedule_and_bits(bm, orc, cuda, layout):
    """4096^3 with the default schedule (its last wave
    holds more than half the pairs, so it stays whole); bit-identical to the
    explicit whole-tile schedule and within tolerance of sampled FP64 oracle
    entries."""
    torch = cuda
    m = n = k = 4096
    a, b, c = bm.alloc_operands(m, n, k, layout, mode=4, seed=0)
    c_whole = torch.empty_like(c)
    _run(bm, a, b, c_whole, layout, bm.SPLIT_NONE, variant=0)
    with bm.Gemm.from_tensors(a, b, c, layout) as g:
        assert g.info()["variant"] == V5
        sched = g.schedule()
        g.launch()
        assert g.status() == (bm.BM_OK, 0)
    res = sched["resident_clusters"]
    assert sched["whole_tiles"] + sched["split_tiles"] == 128, sched
    if 2 * (128 % res) > res:
        assert sched["split_tiles"] == 0, sched
    assert np.array_equal(_bits(c), _bits(c_whole))
    rng = np.random.default_rng(5)
    rows, cols = rng.integers(0, m, 1024), rng.integers(0, n, 1024)
    ha, hb = _bits(a).reshape(-1), _bits(b).reshape(-1)
    lda, ldb = _lds(m, n, k, layout)
    ref = orc.entries_f64(k, layout, ha, lda, hb, ldb, rows, cols)
    bad, merr, _ = orc.check(_bits(c)[cols, rows], ref, k, RTOL, ATOL)
    assert bad == 0, f"{bad} bad samples, max err {merr}"
