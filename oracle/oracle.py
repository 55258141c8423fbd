"""ctypes binding of the CPU oracle (TEST INFRASTRUCTURE ONLY).

Used by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg as the
checker / CPU reference. The product path (best-matmul_b200/) never imports it.

- ``Oracle``: the plain-C restatement in oracle/bm_oracle.c (lib/libbm_oracle.so).
- ``RefLib``: the reference's own host code (host/validation.cuh,
  host/common.cuh of ggbond-x/best-matmul) compiled in place by
  ``make -C oracle ref`` into _ref/libbm_ref.so. Present wherever it was built.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(HERE, "lib", "libbm_oracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libbm_ref.so")

_u16p = ctypes.POINTER(ctypes.c_uint16)
_f64p = ctypes.POINTER(ctypes.c_double)
_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)
_i64 = ctypes.c_int64
_u64 = ctypes.c_uint64
_i32 = ctypes.c_int


def _ptr(a: np.ndarray, typ):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(typ)


def default_threads() -> int:
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except AttributeError:
        return max(1, os.cpu_count() or 1)


class Oracle:
    def __init__(self, path: str = ORACLE_LIB):
        if not os.path.exists(path):
            raise FileNotFoundError(f"oracle not built: {path} (run `make -C oracle`)")
        L = ctypes.CDLL(path)
        L.bmo_half_from_float.restype = ctypes.c_uint16
        L.bmo_half_from_float.argtypes = [ctypes.c_float]
        L.bmo_float_from_half.restype = ctypes.c_float
        L.bmo_float_from_half.argtypes = [ctypes.c_uint16]
        L.bmo_make_inputs.argtypes = [_i32, _i32, _i32, _i32, _i32, _u64, _u16p, _u16p]
        L.bmo_input_value.restype = ctypes.c_uint16
        L.bmo_input_value.argtypes = [_i32, _u64, _i32, _u64, _u64]
        L.bmo_fill.argtypes = [_u16p, _i64, _i64, _i64, _i32, _i64, _i64, _i32, _u64, _i32]
        L.bmo_gemm_entry_f64.restype = ctypes.c_double
        L.bmo_gemm_entry_f64.argtypes = [_i32, _i32, _u16p, _i64, _u16p, _i64, _i32, _i32]
        L.bmo_gemm_entries_f64.argtypes = [_i32, _i32, _u16p, _i64, _u16p, _i64, _i32p, _i32p,
                                           _i64, _f64p, _i32]
        L.bmo_gemm_f32.argtypes = [_i32, _i32, _u16p, _i64, _u16p, _i64, _i32, _i32, _i32, _i32,
                                   _f32p, _i32]
        L.bmo_gemm_exact_int.restype = _i32
        L.bmo_gemm_exact_int.argtypes = [_i32, _i32, _i32, _i32, _u16p, _u16p, _i32p]
        L.bmo_check.restype = _i64
        L.bmo_check.argtypes = [_u16p, _f64p, _i64, _i32, ctypes.c_double, ctypes.c_double,
                                _f64p, ctypes.POINTER(_i64)]
        L.bmo_validate_sampled.restype = _i32
        L.bmo_validate_sampled.argtypes = [_i32, _i32, _i32, _i32, _u16p, _i64, _u16p, _i64,
                                           _u16p, _i64, _f64p, _f64p]
        self.L = L

    # -- FP16
    def half(self, f: float) -> int:
        return self.L.bmo_half_from_float(f)

    def to_float(self, h: int) -> float:
        return self.L.bmo_float_from_half(h)

    # -- inputs
    def make_inputs(self, m, n, k, layout, mode, seed=0):
        """(A, B) as uint16 bit patterns in physical order (GemmBuffers order)."""
        a = np.empty(m * k, dtype=np.uint16)
        b = np.empty(n * k, dtype=np.uint16)
        self.L.bmo_make_inputs(m, n, k, 1 if layout.upper() == "NT" else 0, mode, seed,
                               _ptr(a, _u16p), _ptr(b, _u16p))
        return a, b

    def fill(self, rows, cols, ld, row_major, row0, full_ld, mode, seed, matrix_id):
        n = (rows * ld) if row_major else (cols * ld)
        out = np.zeros(n, dtype=np.uint16)
        self.L.bmo_fill(_ptr(out, _u16p), rows, cols, ld, 1 if row_major else 0, row0, full_ld,
                        mode, seed, matrix_id)
        return out

    # -- reference GEMM
    def entry_f64(self, k, layout, a, lda, b, ldb, row, col) -> float:
        return self.L.bmo_gemm_entry_f64(k, 1 if layout.upper() == "NT" else 0, _ptr(a, _u16p),
                                         lda, _ptr(b, _u16p), ldb, row, col)

    def entries_f64(self, k, layout, a, lda, b, ldb, rows, cols, threads=None) -> np.ndarray:
        rows = np.ascontiguousarray(rows, dtype=np.int32)
        cols = np.ascontiguousarray(cols, dtype=np.int32)
        out = np.empty(rows.size, dtype=np.float64)
        self.L.bmo_gemm_entries_f64(k, 1 if layout.upper() == "NT" else 0, _ptr(a, _u16p), lda,
                                    _ptr(b, _u16p), ldb, _ptr(rows, _i32p), _ptr(cols, _i32p),
                                    rows.size, _ptr(out, _f64p), threads or default_threads())
        return out

    def gemm_f32(self, k, layout, a, lda, b, ldb, row0, rows, col0, cols, threads=None):
        """FP32-accumulate block, returned column-major as a (cols, rows) array."""
        out = np.empty(rows * cols, dtype=np.float32)
        self.L.bmo_gemm_f32(k, 1 if layout.upper() == "NT" else 0, _ptr(a, _u16p), lda,
                            _ptr(b, _u16p), ldb, row0, rows, col0, cols, _ptr(out, _f32p),
                            threads or default_threads())
        return out.reshape(cols, rows)

    def exact_int(self, m, n, k, layout, a, b):
        out = np.empty(m * n, dtype=np.int32)
        rc = self.L.bmo_gemm_exact_int(m, n, k, 1 if layout.upper() == "NT" else 0,
                                       _ptr(a, _u16p), _ptr(b, _u16p), _ptr(out, _i32p))
        return None if rc != 0 else out.reshape(n, m)

    def check(self, c_bits: np.ndarray, ref: np.ndarray, k: int, rtol=1e-2, atol=2e-3):
        """Count of |c - ref| > rtol*|ref| + atol*sqrt(K/4096), max error, worst index."""
        c_bits = np.ascontiguousarray(c_bits.reshape(-1), dtype=np.uint16)
        ref = np.ascontiguousarray(ref.reshape(-1), dtype=np.float64)
        assert c_bits.size == ref.size
        merr = ctypes.c_double(0.0)
        worst = _i64(-1)
        bad = self.L.bmo_check(_ptr(c_bits, _u16p), _ptr(ref, _f64p), c_bits.size, k, rtol, atol,
                               ctypes.byref(merr), ctypes.byref(worst))
        return int(bad), merr.value, worst.value

    def validate_sampled(self, m, n, k, layout, a, lda, b, ldb, c, ldc):
        merr = ctypes.c_double(0.0)
        chk = ctypes.c_double(0.0)
        rc = self.L.bmo_validate_sampled(m, n, k, 1 if layout.upper() == "NT" else 0,
                                         _ptr(a, _u16p), lda, _ptr(b, _u16p), ldb,
                                         _ptr(c, _u16p), ldc, ctypes.byref(merr), ctypes.byref(chk))
        return rc, merr.value, chk.value


class RefLib:
    """The reference's own host code, compiled from its headers (oracle/_ref)."""

    def __init__(self, path: str = REF_LIB):
        if not os.path.exists(path):
            raise FileNotFoundError(f"reference shim not built: {path} (run `make -C oracle ref`)")
        L = ctypes.CDLL(path)
        vp = ctypes.c_void_p
        L.bmref_create.restype = vp
        L.bmref_create.argtypes = [_i32, _i32, _i32, ctypes.c_char, ctypes.c_char, _i32]
        L.bmref_create_from.restype = vp
        L.bmref_create_from.argtypes = [_i32, _i32, _i32, ctypes.c_char, ctypes.c_char, _u16p, _u16p]
        L.bmref_export.argtypes = [vp, _u16p, _u16p]
        for f in ("bmref_a_index", "bmref_b_index", "bmref_c_index"):
            getattr(L, f).restype = _i64
            getattr(L, f).argtypes = [vp, _i32, _i32]
        L.bmref_entry.restype = ctypes.c_double
        L.bmref_entry.argtypes = [vp, _i32, _i32]
        L.bmref_entries.argtypes = [vp, _i32p, _i32p, _i64, _f64p, _i32]
        L.bmref_destroy.argtypes = [vp]
        self.L = L

    def problem(self, m, n, k, layout, mode=None, a=None, b=None):
        return RefProblem(self, m, n, k, layout, mode, a, b)


class RefProblem:
    def __init__(self, lib: RefLib, m, n, k, layout, mode, a, b):
        self.lib, self.m, self.n, self.k, self.layout = lib, m, n, k, layout.upper()
        ta, tb = self.layout[0].encode(), self.layout[1].encode()
        if mode is not None:
            self.h = lib.L.bmref_create(m, n, k, ta, tb, mode)
        else:
            self.h = lib.L.bmref_create_from(m, n, k, ta, tb, _ptr(a, _u16p), _ptr(b, _u16p))

    def export(self):
        a = np.empty(self.m * self.k, dtype=np.uint16)
        b = np.empty(self.n * self.k, dtype=np.uint16)
        self.lib.L.bmref_export(self.h, _ptr(a, _u16p), _ptr(b, _u16p))
        return a, b

    def entry(self, row, col) -> float:
        return self.lib.L.bmref_entry(self.h, row, col)

    def entries(self, rows, cols, threads=None) -> np.ndarray:
        rows = np.ascontiguousarray(rows, dtype=np.int32)
        cols = np.ascontiguousarray(cols, dtype=np.int32)
        out = np.empty(rows.size, dtype=np.float64)
        self.lib.L.bmref_entries(self.h, _ptr(rows, _i32p), _ptr(cols, _i32p), rows.size,
                                 _ptr(out, _f64p), threads or default_threads())
        return out

    def index(self, which, i, j) -> int:
        return getattr(self.lib.L, f"bmref_{which}_index")(self.h, i, j)

    def close(self):
        if self.h:
            self.lib.L.bmref_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
