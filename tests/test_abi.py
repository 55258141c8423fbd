"""C-ABI surface of lib/libbmgemm.so, checked without a GPU."""
from __future__ import annotations

import ctypes

import pytest


def test_library_exports_every_header_symbol(bm):
    lib = bm.load()
    names = bm.header_functions()
    assert "bm_gemm_prepare" in names and "bm_gemm_launch" in names
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_interface_version(bm):
    assert bm.interface_version() == 1  # reference benchmark_host.cu:10


def test_error_strings_and_variant_names(bm):
    for code in range(0, 10):
        assert bm.error_string(code)
    assert bm.error_string(1234) == "unknown error"
    for v in bm.VARIANTS:
        assert bm.variant_name(v).startswith("sm100_tcgen05_")
    assert bm.variant_name(99) == "unknown"


@pytest.mark.parametrize("layout", ["NT", "TN"])
def test_check_accepts_reference_shapes(bm, layout):
    for s in (512, 1024, 4096, 8192, 16384):
        assert bm.check(s, s, s, layout) == bm.BM_OK
    assert bm.check(128, 28672, 8192, "TN") == bm.BM_OK
    assert bm.check(8192, 8192, 28672, "TN") == bm.BM_OK


def test_check_rejects_like_the_reference(bm):
    # host/driver.cuh:97-100: M, N, K > 0
    assert bm.check(0, 64, 64, "NT") == bm.BM_ERR_INVALID_ARGUMENT
    assert bm.check(64, -1, 64, "NT") == bm.BM_ERR_INVALID_ARGUMENT
    # host/driver.cuh:101-105: only NT and TN
    assert bm.check(64, 64, 64, "NN") == bm.BM_ERR_UNSUPPORTED_LAYOUT
    assert bm.check(64, 64, 64, "TT") == bm.BM_ERR_UNSUPPORTED_LAYOUT
    # host/driver.cuh:106-113: element counts <= INT_MAX
    assert bm.check(65536, 65536, 64, "NT") == bm.BM_ERR_SIZE_LIMIT
    assert bm.check(32768, 32768, 32768, "NT") == bm.BM_OK  # 2^30 elements
    # tma_wgmma_adapter.cuh:134-141 (strict mode): tile multiples
    assert bm.check(384, 512, 512, "NT", strict=True, variant=1) == bm.BM_ERR_TILE_DIVISIBILITY
    assert bm.check(512, 512, 96, "TN", strict=True, variant=1) == bm.BM_ERR_TILE_DIVISIBILITY
    assert bm.check(512, 512, 512, "TN", strict=True, variant=1) == bm.BM_OK
    assert bm.check(384, 512, 512, "NT", strict=True, variant=2) == bm.BM_OK


def test_check_alignment_rules(bm):
    # TMA needs 16-byte row pitches: NT leading dims are M and N, TN's are K.
    assert bm.check(100, 64, 64, "NT") == bm.BM_ERR_ALIGNMENT
    assert bm.check(64, 64, 100, "NT") == bm.BM_OK
    assert bm.check(64, 64, 100, "TN") == bm.BM_ERR_ALIGNMENT
    assert bm.check(64, 100, 64, "TN") == bm.BM_OK  # N is no leading dimension in TN
    assert bm.check(64, 100, 64, "NT") == bm.BM_ERR_ALIGNMENT
    assert bm.check(200, 136, 72, "TN") == bm.BM_OK  # ragged but aligned
    assert bm.check(64, 64, 64, "TN", a_ptr=18) == bm.BM_ERR_ALIGNMENT
    assert bm.check(64, 64, 64, "TN", lda=60) == bm.BM_ERR_INVALID_ARGUMENT  # lda < K
    assert bm.check(64, 64, 64, "TN", lda=72) == bm.BM_OK
    assert bm.check(64, 64, 64, "TN", c_ptr=0) == bm.BM_ERR_INVALID_ARGUMENT
    assert bm.check(64, 64, 64, "TN", variant=42) == bm.BM_ERR_VARIANT


def test_prepare_rejects_without_touching_gpu(bm):
    lib = bm.load()
    d = bm.make_desc(64, 64, 64, "NN", 16, 16, 16)
    h = ctypes.c_void_p()
    assert lib.bm_gemm_prepare(ctypes.byref(d), ctypes.byref(h)) == bm.BM_ERR_UNSUPPORTED_LAYOUT
    assert not h.value
    assert lib.bm_gemm_prepare(None, ctypes.byref(h)) == bm.BM_ERR_INVALID_ARGUMENT
    assert lib.bm_gemm_launch(None, None) == bm.BM_ERR_INVALID_ARGUMENT
    assert lib.bm_gemm_query(None, None) == bm.BM_ERR_INVALID_ARGUMENT
    lib.bm_gemm_destroy(None)  # no-op


def test_missing_library_fails_loudly(bm, monkeypatch, tmp_path):
    monkeypatch.setattr(bm, "_lib", None)
    monkeypatch.setattr(bm, "LIB_PATH", str(tmp_path / "libbmgemm.so"))
    with pytest.raises(bm.BmGemmError):
        bm.load()
