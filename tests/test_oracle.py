"""The CPU oracle, pinned against the reference's own code.

Golden vectors (tests/golden/reference_golden.json) were produced by the
reference's host/common.cuh + host/validation.cuh compiled in place
(tests/golden/make_golden.py). Where the reference shim is built (this
container), the oracle is also compared with it live on extra shapes.
"""
from __future__ import annotations

import hashlib
import json
import math
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reference_golden.json")


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _lds(m, n, k, layout):
    return (m, n) if layout == "NT" else (k, k)


@pytest.fixture(scope="module")
def golden():
    with open(GOLDEN) as f:
        return json.load(f)


def test_half_rounding_matches_ieee(orc):
    rng = np.random.default_rng(1)
    xs = np.concatenate([rng.standard_normal(4000).astype(np.float32) * s
                         for s in (1e-8, 3e-7, 6e-5, 1e-2, 1.0, 300.0, 6e4)])
    special = np.array([0.0, -0.0, 65504.0, 65519.996, 65520.0, 1e9, -1e9, 2.9802322e-08,
                        2.9802326e-08, 5.9604645e-08, 1e-30], dtype=np.float32)
    xs = np.concatenate([xs, special])
    with np.errstate(over="ignore"):
        expect = xs.astype(np.float16).view(np.uint16)
    got = np.array([orc.half(float(v)) for v in xs], dtype=np.uint16)
    assert np.array_equal(got, expect)


def test_half_to_float_all_patterns(orc):
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    expect = bits.view(np.float16).astype(np.float32)
    got = np.array([orc.to_float(int(b)) for b in bits], dtype=np.float32)
    finite = np.isfinite(expect)
    assert np.array_equal(got[finite], expect[finite])
    assert np.array_equal(np.isnan(got), np.isnan(expect))
    assert np.array_equal(np.isinf(got), np.isinf(expect))


def test_inputs_match_reference_golden(orc, golden):
    for case in golden["reference_cases"]:
        m, n, k, layout, mode = case["m"], case["n"], case["k"], case["layout"], case["mode"]
        a, b = orc.make_inputs(m, n, k, layout, mode)
        assert _sha(a) == case["sha_a"], (m, n, k, layout, mode)
        assert _sha(b) == case["sha_b"], (m, n, k, layout, mode)
        assert a[:8].tolist() == case["a_head"]


def test_entries_match_reference_golden(orc, golden):
    for case in golden["reference_cases"]:
        m, n, k, layout, mode = case["m"], case["n"], case["k"], case["layout"], case["mode"]
        a, b = orc.make_inputs(m, n, k, layout, mode)
        lda, ldb = _lds(m, n, k, layout)
        got = orc.entries_f64(k, layout, a, lda, b, ldb, case["rows"], case["cols"], threads=1)
        assert got.tolist() == case["entries"], (m, n, k, layout, mode)  # bit-exact FP64
        if "full_sha_f64" in case:
            rows = np.repeat(np.arange(m), n)
            cols = np.tile(np.arange(n), m)
            full = orc.entries_f64(k, layout, a, lda, b, ldb, rows, cols, threads=1)
            assert _sha(full.astype(np.float64)) == case["full_sha_f64"]


def test_index_functions_match_reference_golden(orc, golden):
    from oracle import Oracle  # noqa: F401  (index functions live in the C library)
    import ctypes
    L = orc.L
    L.bmo_a_index.restype = ctypes.c_int64
    L.bmo_a_index.argtypes = [ctypes.c_int, ctypes.c_int64, ctypes.c_int, ctypes.c_int]
    L.bmo_b_index.restype = ctypes.c_int64
    L.bmo_b_index.argtypes = [ctypes.c_int, ctypes.c_int64, ctypes.c_int, ctypes.c_int]
    for case in golden["reference_cases"]:
        m, n, k, layout = case["m"], case["n"], case["k"], case["layout"]
        nt = 1 if layout == "NT" else 0
        lda, ldb = _lds(m, n, k, layout)
        a_pts = ((0, 0), (m - 1, 0), (0, k - 1), (m // 2, k // 3))
        b_pts = ((0, 0), (n - 1, 0), (0, k - 1), (n // 2, k // 3))
        c_pts = ((0, 0), (m - 1, 0), (0, n - 1), (m // 2, n // 3))
        assert [L.bmo_a_index(nt, lda, r, p) for r, p in a_pts] == case["index"]["a"]
        assert [L.bmo_b_index(nt, ldb, c, p) for c, p in b_pts] == case["index"]["b"]
        assert [r + c * m for r, c in c_pts] == case["index"]["c"]


def test_generator_golden(orc, golden):
    for case in golden["generator_cases"]:
        a, b = orc.make_inputs(case["m"], case["n"], case["k"], case["layout"], case["mode"],
                               seed=case["seed"])
        assert _sha(a) == case["sha_a"]
        assert _sha(b) == case["sha_b"]


def test_generator_is_layout_independent_and_shardable(orc):
    """Modes 4/5 depend on the logical (row, k) only: NT and TN hold the same
    logical matrix, and any row block regenerates identically."""
    m, n, k = 96, 64, 80
    for mode in (4, 5):
        a_nt, b_nt = orc.make_inputs(m, n, k, "NT", mode, seed=7)
        a_tn, b_tn = orc.make_inputs(m, n, k, "TN", mode, seed=7)
        assert np.array_equal(a_nt.reshape(k, m).T, a_tn.reshape(m, k))
        assert np.array_equal(b_nt.reshape(k, n).T, b_tn.reshape(n, k))
        blk = orc.fill(32, k, k, 1, 40, k, mode, 7, 0)  # rows 40..71, row-major
        assert np.array_equal(blk.reshape(32, k), a_tn.reshape(m, k)[40:72])
        blk_cm = orc.fill(32, k, 32, 0, 40, m, mode, 7, 0)  # same rows, column-major ld 32
        assert np.array_equal(blk_cm.reshape(k, 32).T, a_tn.reshape(m, k)[40:72])


def test_generator_distributions(orc):
    a, _ = orc.make_inputs(512, 8, 512, "TN", 4, seed=0)
    v = a.view(np.float16).astype(np.float64)
    assert v.min() >= -1.0 and v.max() <= 1.0
    assert abs(v.mean()) < 0.01 and abs(v.std() - 1 / math.sqrt(3)) < 0.01
    a, _ = orc.make_inputs(512, 8, 512, "TN", 5, seed=0)
    v = a.view(np.float16).astype(np.float64)
    assert abs(v.mean()) < 5e-4 and abs(v.std() - 0.02) < 5e-4


def test_known_answers(orc):
    """Reference golden behaviour: mode 1 -> C = K everywhere; mode 0 -> 0;
    integer modes are exact (tests/full_output_validation.cu:84-101)."""
    m, n, k = 64, 48, 136
    for layout in ("NT", "TN"):
        lda, ldb = _lds(m, n, k, layout)
        a, b = orc.make_inputs(m, n, k, layout, 1)
        c = orc.gemm_f32(k, layout, a, lda, b, ldb, 0, m, 0, n)
        assert np.all(c == k)
        a, b = orc.make_inputs(m, n, k, layout, 0)
        assert np.all(orc.gemm_f32(k, layout, a, lda, b, ldb, 0, m, 0, n) == 0)
        for mode in (2, 3):
            a, b = orc.make_inputs(m, n, k, layout, mode)
            exact = orc.exact_int(m, n, k, layout, a, b)
            assert exact is not None
            f32 = orc.gemm_f32(k, layout, a, lda, b, ldb, 0, m, 0, n)
            assert np.array_equal(f32, exact.astype(np.float32))
            rows = np.repeat(np.arange(m), n)
            cols = np.tile(np.arange(n), m)
            f64 = orc.entries_f64(k, layout, a, lda, b, ldb, rows, cols)
            assert np.array_equal(f64.reshape(m, n).T, exact.astype(np.float64))


def test_exact_int_rejects_fp16_overflow(orc):
    m, n, k = 8, 8, 4096
    a, b = orc.make_inputs(m, n, k, "TN", 1)
    assert orc.exact_int(m, n, k, "TN", a, b) is None  # partial sums pass 2048


def test_check_tolerance_formula(orc):
    k = 16384
    ref = np.array([0.0, 1.0, -100.0, 1e-3], dtype=np.float64)
    atol = 2e-3 * math.sqrt(k / 4096)
    tol = 1e-2 * np.abs(ref) + atol
    inside = (ref + 0.9 * tol).astype(np.float16).view(np.uint16)
    bad, _, _ = orc.check(inside, ref.astype(np.float16).astype(np.float64), k)
    assert bad == 0
    outside = (ref + 3 * tol).astype(np.float16).view(np.uint16)
    bad, _, _ = orc.check(outside, ref, k)
    assert bad == 4


def test_planted_error_is_caught(orc):
    """A mistake planted in an otherwise correct output (on the CPU) must be
    reported by the checker, including a NaN."""
    m, n, k = 64, 64, 128
    a, b = orc.make_inputs(m, n, k, "TN", 4)
    ref = orc.gemm_f32(k, "TN", a, k, b, k, 0, m, 0, n).astype(np.float64)
    c = ref.astype(np.float16).view(np.uint16).copy()
    assert orc.check(c, ref, k)[0] == 0
    c2 = c.copy()
    c2.reshape(-1)[1234] ^= 0x0400  # flip an exponent bit
    assert orc.check(c2, ref, k)[0] == 1
    c3 = c.copy()
    c3.reshape(-1)[77] = 0x7E00  # NaN
    assert orc.check(c3, ref, k)[0] == 1


def test_validate_sampled_restatement(orc):
    m, n, k = 128, 96, 64
    for layout in ("NT", "TN"):
        lda, ldb = _lds(m, n, k, layout)
        a, b = orc.make_inputs(m, n, k, layout, 2)
        ref = orc.gemm_f32(k, layout, a, lda, b, ldb, 0, m, 0, n)
        c = ref.astype(np.float16).view(np.uint16).copy()
        rc, merr, chk = orc.validate_sampled(m, n, k, layout, a, lda, b, ldb, c, m)
        assert rc == 0 and merr == 0.0 and chk == float(ref.sum())
        c[(n - 1) // 3, (m - 1) // 3] = np.float16(1000.0).view(np.uint16)  # sample (row 42, col 31)
        rc, _, _ = orc.validate_sampled(m, n, k, layout, a, lda, b, ldb, c, m)
        assert rc != 0


@pytest.mark.parametrize("layout", ["NT", "TN"])
def test_live_against_reference(orc, reflib, layout):
    """Oracle vs the reference's own compiled code on shapes beyond the fixtures."""
    rng = np.random.default_rng(3)
    for (m, n, k) in ((200, 136, 72), (512, 64, 300)):
        for mode in (2, 3):
            a, b = orc.make_inputs(m, n, k, layout, mode)
            p = reflib.problem(m, n, k, layout, mode=mode)
            ra, rb = p.export()
            assert np.array_equal(a, ra) and np.array_equal(b, rb)
            rows = rng.integers(0, m, 500)
            cols = rng.integers(0, n, 500)
            lda, ldb = _lds(m, n, k, layout)
            assert np.array_equal(orc.entries_f64(k, layout, a, lda, b, ldb, rows, cols),
                                  p.entries(rows, cols))
        a, b = orc.make_inputs(m, n, k, layout, 4, seed=11)
        p = reflib.problem(m, n, k, layout, a=a, b=b)
        rows = rng.integers(0, m, 300)
        cols = rng.integers(0, n, 300)
        lda, ldb = _lds(m, n, k, layout)
        assert np.array_equal(orc.entries_f64(k, layout, a, lda, b, ldb, rows, cols),
                              p.entries(rows, cols))
