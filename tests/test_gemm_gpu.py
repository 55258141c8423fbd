"""GPU parity of the sm_100a GEMM against the CPU oracle, through the C ABI.

Tolerance on every checked element:
    |c - ref| <= 1e-2 * |ref| + 2e-3 * sqrt(K / 4096)
with ref the oracle's FP32-accumulate GEMM (full outputs) or its FP64
reference_gemm_entry restatement (sampled outputs of large shapes).
Integer inputs are checked bit for bit (tests/full_output_validation.cu pattern).
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-2, 2e-3


def _lds(m, n, k, layout):
    return (m, n) if layout == "NT" else (k, k)


def _to_dev(torch, a_bits, b_bits, m, n, k, layout):
    if layout == "NT":
        a = torch.from_numpy(a_bits.view(np.float16).reshape(k, m).copy()).cuda()
        b = torch.from_numpy(b_bits.view(np.float16).reshape(k, n).copy()).cuda()
    else:
        a = torch.from_numpy(a_bits.view(np.float16).reshape(m, k).copy()).cuda()
        b = torch.from_numpy(b_bits.view(np.float16).reshape(n, k).copy()).cuda()
    c = torch.full((n, m), float("nan"), dtype=torch.float16, device="cuda")
    return a, b, c


def _bits(t):
    return t.cpu().numpy().view(np.uint16)


def _run(bm, a, b, c, layout, variant, launches=1):
    with bm.Gemm.from_tensors(a, b, c, layout, variant=variant) as g:
        for _ in range(launches):
            g.launch()
        rc, bits = g.status()
        info = g.info()
    assert rc == bm.BM_OK, f"kernel status {rc}, device bits {bits:#x}"
    return info


def _describe_mismatch(got, want, m, n, tile_m, tile_n):
    bad = np.argwhere(got != want)
    cols, rows = bad[:, 0], bad[:, 1]
    return (f"{len(bad)} of {m * n} differ; rows {rows.min()}..{rows.max()}, cols "
            f"{cols.min()}..{cols.max()}; tiles (m,n) {sorted(set(zip((rows // tile_m).tolist(), (cols // tile_n).tolist())))[:8]}; "
            f"first (row {rows[0]}, col {cols[0]}): got {got[cols[0], rows[0]]} want {want[cols[0], rows[0]]}")


# ----------------------------------------------------------------- inputs
@pytest.mark.parametrize("mode", [0, 1, 3, 4, 5])
def test_device_fill_matches_oracle(bm, orc, cuda, mode):
    torch = cuda
    rows, cols = 200, 72
    for row_major in (True, False):
        ld = cols + 8 if row_major else rows + 8
        n_el = rows * ld if row_major else cols * ld
        t = torch.zeros(n_el, dtype=torch.float16, device="cuda")
        bm.fill(t, rows, cols, row_major, mode, seed=5, matrix_id=1, row0=40, full_ld=ld + 40,
                ld=ld)
        got = _bits(t)
        want = orc.fill(rows, cols, ld, row_major, 40, ld + 40, mode, 5, 1)
        assert np.array_equal(got, want)


@pytest.mark.parametrize("layout", ["NT", "TN"])
def test_alloc_operands_match_oracle_inputs(bm, orc, cuda, layout):
    m, n, k = 256, 128, 192
    a, b, _ = bm.alloc_operands(m, n, k, layout, mode=4, seed=3)
    ea, eb = orc.make_inputs(m, n, k, layout, 4, seed=3)
    assert np.array_equal(_bits(a).reshape(-1), ea)
    assert np.array_equal(_bits(b).reshape(-1), eb)


# ----------------------------------------------------------------- parity
@pytest.mark.parametrize("variant", [1, 2, 3, 4, 5])
@pytest.mark.parametrize("layout", ["NT", "TN"])
def test_parity_512_uniform(bm, orc, cuda, layout, variant):
    """512^3, uniform[-1,1] seed 0, full output."""
    m = n = k = 512
    a, b, c = bm.alloc_operands(m, n, k, layout, mode=4, seed=0)
    c.fill_(float("nan"))
    _run(bm, a, b, c, layout, variant)
    ea, eb = orc.make_inputs(m, n, k, layout, 4, seed=0)
    lda, ldb = _lds(m, n, k, layout)
    ref = orc.gemm_f32(k, layout, ea, lda, eb, ldb, 0, m, 0, n).astype(np.float64)
    bad, merr, worst = orc.check(_bits(c), ref, k, RTOL, ATOL)
    assert bad == 0, f"{bad} outside tolerance, max err {merr}, worst {worst}"


def _ktile_set(stages):
    return sorted({1, 2, stages - 1, stages, stages + 1, 3 * stages + 1} - {0})


@pytest.mark.parametrize("variant", [1, 2, 3, 4, 5])
@pytest.mark.parametrize("layout", ["NT", "TN"])
def test_full_output_exact_integers(bm, orc, cuda, layout, variant):
    """tests/full_output_validation.cu:54-152 on the new kernel: M = 2 tiles,
    N = 2 tiles, K-tile counts around the pipeline depth (phase wrap),
    reference input modes 0..3, NaN-prefilled C, two launches, every element
    compared bit for bit with the FP16 rounding of the exact integer result."""
    torch = cuda
    tile_m, tile_n, stages = bm.VARIANT_TILES[variant]
    m, n = 2 * tile_m, 2 * tile_n
    for kt in _ktile_set(stages):
        k = kt * 64
        lda, ldb = _lds(m, n, k, layout)
        for mode in (0, 1, 2, 3):
            ea, eb = orc.make_inputs(m, n, k, layout, mode)
            a, b, c = _to_dev(torch, ea, eb, m, n, k, layout)
            _run(bm, a, b, c, layout, variant, launches=2)
            exact = orc.gemm_f32(k, layout, ea, lda, eb, ldb, 0, m, 0, n)  # exact: integers < 2^24
            want = exact.astype(np.float16).view(np.uint16)
            got = _bits(c)
            assert np.array_equal(got, want), (
                f"{layout} variant {variant} K tiles {kt} mode {mode}: "
                + _describe_mismatch(got, want, m, n, tile_m, tile_n))


@pytest.mark.parametrize("layout", ["NT", "TN"])
@pytest.mark.parametrize("shape", [(200, 136, 72), (264, 520, 1000), (136, 8, 64), (8, 264, 8)])
def test_ragged_shapes(bm, orc, cuda, layout, shape):
    """Shapes that are not tile multiples: TMA zero-fills loads past the edge
    and clips stores (beyond the reference, which rejects them)."""
    m, n, k = shape
    if bm.check(m, n, k, layout) != bm.BM_OK:
        pytest.skip("leading dimension not a multiple of 8 for this layout")
    for variant in (1, 2, 3, 4, 5):
        a, b, c = bm.alloc_operands(m, n, k, layout, mode=4, seed=9)
        c.fill_(float("nan"))
        _run(bm, a, b, c, layout, variant)
        ea, eb = orc.make_inputs(m, n, k, layout, 4, seed=9)
        lda, ldb = _lds(m, n, k, layout)
        ref = orc.gemm_f32(k, layout, ea, lda, eb, ldb, 0, m, 0, n).astype(np.float64)
        bad, merr, worst = orc.check(_bits(c), ref, k, RTOL, ATOL)
        assert bad == 0, f"variant {variant}: {bad} bad, max err {merr}, worst {worst}"


@pytest.mark.parametrize("layout", ["NT", "TN"])
def test_strided_leading_dimensions(bm, orc, cuda, layout):
    """lda/ldb/ldc larger than the reference defaults (sub-matrix views)."""
    torch = cuda
    m, n, k = 256, 256, 128
    ea, eb = orc.make_inputs(m, n, k, layout, 4, seed=2)
    pad = 64
    if layout == "NT":
        a = torch.zeros((k, m + pad), dtype=torch.float16, device="cuda")
        b = torch.zeros((k, n + pad), dtype=torch.float16, device="cuda")
        a[:, :m] = torch.from_numpy(ea.view(np.float16).reshape(k, m)).cuda()
        b[:, :n] = torch.from_numpy(eb.view(np.float16).reshape(k, n)).cuda()
        lda, ldb = m + pad, n + pad
    else:
        a = torch.zeros((m, k + pad), dtype=torch.float16, device="cuda")
        b = torch.zeros((n, k + pad), dtype=torch.float16, device="cuda")
        a[:, :k] = torch.from_numpy(ea.view(np.float16).reshape(m, k)).cuda()
        b[:, :k] = torch.from_numpy(eb.view(np.float16).reshape(n, k)).cuda()
        lda, ldb = k + pad, k + pad
    c = torch.full((n, m + pad), float("nan"), dtype=torch.float16, device="cuda")
    with bm.Gemm(m, n, k, layout, a.data_ptr(), b.data_ptr(), c.data_ptr(), lda, ldb,
                 m + pad) as g:
        g.launch()
        assert g.status()[0] == bm.BM_OK
    got = _bits(c)
    assert np.all(np.isnan(c[:, m:].float().cpu().numpy())), "wrote outside the C view"
    lda0, ldb0 = _lds(m, n, k, layout)
    ref = orc.gemm_f32(k, layout, ea, lda0, eb, ldb0, 0, m, 0, n).astype(np.float64)
    bad, merr, _ = orc.check(np.ascontiguousarray(got[:, :m]), ref, k, RTOL, ATOL)
    assert bad == 0, f"{bad} bad, max err {merr}"


@pytest.mark.parametrize("layout", ["NT", "TN"])
@pytest.mark.parametrize("size", [4096, 8192])
def test_large_square_sampled(bm, orc, cuda, layout, size):
    """BASELINE configs[1..2] sizes: sampled FP64 reference entries (4x4 grid,
    corners of every 256-tile row/col band and 512 random points)."""
    torch = cuda
    m = n = k = size
    a, b, c = bm.alloc_operands(m, n, k, layout, mode=4, seed=0)
    c.fill_(float("nan"))
    info = _run(bm, a, b, c, layout, 0)
    assert info["variant"] in bm.VARIANTS
    ha, hb, hc = _bits(a).reshape(-1), _bits(b).reshape(-1), _bits(c)
    rng = np.random.default_rng(size)
    rows = list(rng.integers(0, m, 512))
    cols = list(rng.integers(0, n, 512))
    for t in range(0, m, 256):
        rows += [t, t + 255, t + 128]
        cols += [(t * 7) % n, (t * 13 + 255) % n, t]
    for r in range(4):
        for q in range(4):
            rows.append((m - 1) * r // 3)
            cols.append((n - 1) * q // 3)
    rows, cols = np.array(rows), np.array(cols)
    lda, ldb = _lds(m, n, k, layout)
    ref = orc.entries_f64(k, layout, ha, lda, hb, ldb, rows, cols)
    got = hc[cols, rows]
    bad, merr, worst = orc.check(got, ref, k, RTOL, ATOL)
    assert bad == 0, f"{bad} bad samples, max err {merr}, worst sample {worst}"
    assert not torch.isnan(c).any().item()


@pytest.mark.parametrize("layout", ["NT", "TN"])
def test_all_ones_full_output_large(bm, cuda, layout):
    """Known answer at full size: mode 1 inputs give C = K in every element
    (exact in FP16 for K = 8192); catches any missing or misplaced tile."""
    torch = cuda
    m = n = k = 8192
    a, b, c = bm.alloc_operands(m, n, k, layout, mode=1)
    c.fill_(float("nan"))
    _run(bm, a, b, c, layout, 0)
    assert torch.all(c == float(k)).item()


def test_non_default_stream_and_repeat(bm, orc, cuda):
    torch = cuda
    m = n = k = 1024
    a, b, c = bm.alloc_operands(m, n, k, "TN", mode=4, seed=1)
    s = torch.cuda.Stream()
    with bm.Gemm.from_tensors(a, b, c, "TN") as g:
        for _ in range(5):
            g.launch(s)
        s.synchronize()
        assert g.status()[0] == bm.BM_OK
    ea, eb = orc.make_inputs(m, n, k, "TN", 4, seed=1)
    rows = np.arange(0, m, 7)
    cols = (rows * 5) % n
    ref = orc.entries_f64(k, "TN", ea, k, eb, k, rows, cols)
    assert orc.check(_bits(c)[cols, rows], ref, k)[0] == 0


def test_forced_wait_expires_and_reports(bm, cuda):
    """Failure detection without a GPU fault: the epilogue waits on a barrier
    nothing signals, the bounded wait expires after 1 ms, the status word
    reports it, and the context stays usable for the next GEMM."""
    torch = cuda
    m, n, k = 128, 256, 64
    a, b, c = bm.alloc_operands(m, n, k, "TN", mode=1)
    c.fill_(float("nan"))
    with bm.Gemm.from_tensors(a, b, c, "TN", variant=bm.VARIANT_1CTA_128x256) as g:
        g.set_debug(1_000_000, bm.DEBUG_EPILOGUE_WAITS_NEVER)
        g.launch()
        rc, bits = g.status()
        assert rc == bm.BM_ERR_DEVICE_TIMEOUT
        assert bits & (1 << 4), f"bits {bits:#x}"
    assert torch.isnan(c).all().item(), "the aborted epilogue must not have stored C"
    with bm.Gemm.from_tensors(a, b, c, "TN", variant=bm.VARIANT_1CTA_128x256) as g:
        g.launch()
        assert g.status() == (bm.BM_OK, 0)
    assert torch.all(c == float(k)).item()


def test_dependent_launches_in_one_stream(bm, cuda):
    """Launches use programmatic dependent launch: the next GEMM's CTAs may be
    scheduled while the previous kernel runs, and must not touch global memory
    before it completes. GEMM 2 reads GEMM 1's output as its A operand, back to
    back on one stream; GEMM 1 is long (K = 4096) but occupies only 2 pairs,
    so GEMM 2's CTAs are resident early. C1 is NaN-prefilled: any early read
    shows up in C2. Values are exact: C1 = 4096 * 2^-12 = 1, C2 = 512."""
    torch = cuda
    m, n1, k1, n2 = 512, 512, 4096, 512
    a1 = torch.ones((k1, m), dtype=torch.float16, device="cuda")
    b1 = torch.full((k1, n1), 2.0 ** -12, dtype=torch.float16, device="cuda")
    c1 = torch.empty((n1, m), dtype=torch.float16, device="cuda")
    b2 = torch.ones((n1, n2), dtype=torch.float16, device="cuda")
    c2 = torch.empty((n2, m), dtype=torch.float16, device="cuda")
    with bm.Gemm.from_tensors(a1, b1, c1, "NT") as g1, bm.Gemm.from_tensors(c1, b2, c2, "NT") as g2:
        for rep in range(8):
            c1.fill_(float("nan"))
            c2.fill_(float("nan"))
            g1.launch()
            g2.launch()
            g1.launch()  # rewrite C1 while the next iteration's fill waits behind it
            torch.cuda.synchronize()
            assert torch.all(c1 == 1.0).item(), f"rep {rep}: C1"
            assert torch.all(c2 == float(n1)).item(), f"rep {rep}: C2 read C1 too early"
        assert g1.status() == (bm.BM_OK, 0) and g2.status() == (bm.BM_OK, 0)
