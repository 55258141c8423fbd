"""Python plumbing over the C ABI of the sm_100a FP16 GEMM (include/bm_gemm.h).

The product is the CUDA library ``lib/libbmgemm.so`` next to this file. This
module only binds it with ctypes and uses PyTorch for device memory and
streams; every GEMM goes through ``bm_gemm_launch``. There is no fallback:
if the library is missing, importing the binding raises ``BmGemmError``.

Layout conventions follow gemm_bench::GemmProblem (reference
host/common.cuh:43-76). For torch tensors that means:

  NT ('N','T'): A stored (K, M) row-major  -> a[m + k*M]
                B stored (K, N) row-major  -> b[n + k*N]
  TN ('T','N'): A stored (M, K) row-major  -> a[m*K + k]
                B stored (N, K) row-major  -> b[n*K + k]
  C (both)    : stored (N, M) row-major    -> c[m + n*M]   (column-major C)
"""
from __future__ import annotations

import ctypes
import os
import re

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libbmgemm.so")
HEADER_PATH = os.path.join(os.path.dirname(_HERE), "include", "bm_gemm.h")

BM_OK = 0
BM_ERR_INVALID_ARGUMENT = 1
BM_ERR_UNSUPPORTED_LAYOUT = 2
BM_ERR_ALIGNMENT = 3
BM_ERR_SIZE_LIMIT = 4
BM_ERR_CUDA = 5
BM_ERR_DEVICE = 6
BM_ERR_DEVICE_TIMEOUT = 7
BM_ERR_VARIANT = 8
BM_ERR_TILE_DIVISIBILITY = 9

VARIANT_AUTO = 0
VARIANT_2CTA_256x256 = 1
VARIANT_1CTA_128x256 = 2
VARIANT_1CTA_128x128 = 3
VARIANT_2CTA_256x128 = 4
VARIANT_2CTA_256x512 = 5
VARIANTS = (1, 2, 3, 4, 5)
# (tile_m, tile_n, stages) per variant
VARIANT_TILES = {1: (256, 256, 6), 2: (128, 256, 4), 3: (128, 128, 6), 4: (256, 128, 6),
                 5: (256, 512, 4)}

DEBUG_EPILOGUE_WAITS_NEVER = 1

SPLIT_NONE = 0
SPLIT_AUTO = 1


class BmGemmError(RuntimeError):
    def __init__(self, code: int, what: str = ""):
        self.code = code
        msg = f"bm_gemm error {code}"
        try:
            msg += f" ({error_string(code)})"
        except Exception:  # library not loadable
            pass
        if what:
            msg = f"{what}: {msg}"
        super().__init__(msg)


class GemmDesc(ctypes.Structure):
    _fields_ = [
        ("m", ctypes.c_int), ("n", ctypes.c_int), ("k", ctypes.c_int),
        ("trans_a", ctypes.c_char), ("trans_b", ctypes.c_char),
        ("a", ctypes.c_void_p), ("b", ctypes.c_void_p), ("c", ctypes.c_void_p),
        ("lda", ctypes.c_int64), ("ldb", ctypes.c_int64), ("ldc", ctypes.c_int64),
        ("variant", ctypes.c_int), ("strict_tiles", ctypes.c_int),
    ]


class ScheduleInfo(ctypes.Structure):
    _fields_ = [
        ("whole_tiles", ctypes.c_int), ("split_tiles", ctypes.c_int),
        ("split_parts", ctypes.c_int), ("split_clusters", ctypes.c_int),
        ("grid_clusters", ctypes.c_int), ("resident_clusters", ctypes.c_int),
        ("split_cols", ctypes.c_int),
    ]


class LaunchInfo(ctypes.Structure):
    _fields_ = [
        ("smem_bytes", ctypes.c_int),
        ("grid", ctypes.c_int * 3), ("block", ctypes.c_int * 3), ("cluster", ctypes.c_int * 3),
        ("variant", ctypes.c_int),
        ("tile_m", ctypes.c_int), ("tile_n", ctypes.c_int), ("tile_k", ctypes.c_int),
        ("stages", ctypes.c_int), ("num_tiles", ctypes.c_int), ("cta_group", ctypes.c_int),
    ]


_lib = None


def load() -> ctypes.CDLL:
    """Load lib/libbmgemm.so (once). Raises BmGemmError if it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise BmGemmError(BM_ERR_CUDA, f"CUDA library missing at {LIB_PATH}; build it with "
                          "`python -c 'import __graft_entry__ as g; g.build()'`")
    lib = ctypes.CDLL(LIB_PATH)
    vp, i32, i64, u32, u64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_uint32, ctypes.c_uint64
    lib.bm_gemm_interface_version.restype = i32
    lib.bm_gemm_error_string.restype = ctypes.c_char_p
    lib.bm_gemm_error_string.argtypes = [i32]
    lib.bm_gemm_variant_name.restype = ctypes.c_char_p
    lib.bm_gemm_variant_name.argtypes = [i32]
    lib.bm_gemm_check.restype = i32
    lib.bm_gemm_check.argtypes = [ctypes.POINTER(GemmDesc)]
    lib.bm_gemm_prepare.restype = i32
    lib.bm_gemm_prepare.argtypes = [ctypes.POINTER(GemmDesc), ctypes.POINTER(vp)]
    lib.bm_gemm_launch.restype = i32
    lib.bm_gemm_launch.argtypes = [vp, vp]
    lib.bm_gemm_query.restype = i32
    lib.bm_gemm_query.argtypes = [vp, ctypes.POINTER(LaunchInfo)]
    lib.bm_gemm_status.restype = i32
    lib.bm_gemm_status.argtypes = [vp, ctypes.POINTER(u32)]
    lib.bm_gemm_set_debug.restype = i32
    lib.bm_gemm_set_debug.argtypes = [vp, u64, u32]
    lib.bm_gemm_set_split.restype = i32
    lib.bm_gemm_set_split.argtypes = [vp, i32]
    lib.bm_gemm_query_schedule.restype = i32
    lib.bm_gemm_query_schedule.argtypes = [vp, ctypes.POINTER(ScheduleInfo)]
    lib.bm_gemm_destroy.restype = None
    lib.bm_gemm_destroy.argtypes = [vp]
    lib.bm_fill_fp16.restype = i32
    lib.bm_fill_fp16.argtypes = [vp, i64, i64, i64, i32, i64, i64, i32, u64, i32, vp]
    _lib = lib
    return lib


def header_functions(path: str = HEADER_PATH) -> list[str]:
    """Names of the functions declared in include/bm_gemm.h."""
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(bm_[a-z0-9_]+)\s*\(", text)))


def error_string(code: int) -> str:
    return load().bm_gemm_error_string(code).decode()


def variant_name(variant: int) -> str:
    return load().bm_gemm_variant_name(variant).decode()


def interface_version() -> int:
    return load().bm_gemm_interface_version()


def _layout(layout: str) -> tuple[bytes, bytes]:
    layout = layout.upper()
    if len(layout) != 2:
        raise ValueError("layout must be 'NT' or 'TN'")
    return layout[0].encode(), layout[1].encode()


def make_desc(m, n, k, layout, a_ptr, b_ptr, c_ptr, lda=0, ldb=0, ldc=0, variant=0,
              strict=False) -> GemmDesc:
    ta, tb = _layout(layout)
    return GemmDesc(m, n, k, ta, tb, a_ptr, b_ptr, c_ptr, lda, ldb, ldc, variant,
                    1 if strict else 0)


def check(m, n, k, layout, a_ptr=16, b_ptr=16, c_ptr=16, lda=0, ldb=0, ldc=0, variant=0,
          strict=False) -> int:
    """bm_gemm_check: validation only, no GPU needed. Returns the status code."""
    d = make_desc(m, n, k, layout, a_ptr, b_ptr, c_ptr, lda, ldb, ldc, variant, strict)
    return load().bm_gemm_check(ctypes.byref(d))


def _stream_handle(stream) -> int | None:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


class Gemm:
    """A prepared GEMM (bm_gemm_prepare); launch() enqueues one run."""

    def __init__(self, m, n, k, layout, a_ptr, b_ptr, c_ptr, lda=0, ldb=0, ldc=0, variant=0,
                 strict=False):
        self._lib = load()
        self.m, self.n, self.k, self.layout = m, n, k, layout.upper()
        self._desc = make_desc(m, n, k, layout, a_ptr, b_ptr, c_ptr, lda, ldb, ldc, variant,
                               strict)
        h = ctypes.c_void_p()
        rc = self._lib.bm_gemm_prepare(ctypes.byref(self._desc), ctypes.byref(h))
        if rc != BM_OK:
            raise BmGemmError(rc, "bm_gemm_prepare")
        self._h = h

    @classmethod
    def from_tensors(cls, a, b, c, layout, variant=0, strict=False):
        """Prepare from torch tensors in the layouts listed in the module docstring."""
        layout = layout.upper()
        if layout == "NT":
            k, m = a.shape
            n = b.shape[1]
            assert b.shape[0] == k
        elif layout == "TN":
            m, k = a.shape
            n = b.shape[0]
            assert b.shape[1] == k
        else:
            raise ValueError("layout must be NT or TN")
        assert tuple(c.shape) == (n, m), "C must be stored (N, M) row-major (column-major C)"
        for t in (a, b, c):
            assert t.is_cuda and t.is_contiguous() and t.dtype.itemsize == 2
        g = cls(m, n, k, layout, a.data_ptr(), b.data_ptr(), c.data_ptr(), variant=variant,
                strict=strict)
        g._keep = (a, b, c)
        return g

    def launch(self, stream=None) -> None:
        rc = self._lib.bm_gemm_launch(self._h, _stream_handle(stream))
        if rc != BM_OK:
            raise BmGemmError(rc, "bm_gemm_launch")

    def info(self) -> dict:
        li = LaunchInfo()
        rc = self._lib.bm_gemm_query(self._h, ctypes.byref(li))
        if rc != BM_OK:
            raise BmGemmError(rc, "bm_gemm_query")
        return {
            "smem_bytes": li.smem_bytes, "grid": tuple(li.grid), "block": tuple(li.block),
            "cluster": tuple(li.cluster), "variant": li.variant,
            "name": variant_name(li.variant), "tile": (li.tile_m, li.tile_n, li.tile_k),
            "stages": li.stages, "num_tiles": li.num_tiles, "cta_group": li.cta_group,
        }

    def set_split(self, mode: int) -> None:
        """bm_gemm_set_split: SPLIT_AUTO (default) or SPLIT_NONE."""
        rc = self._lib.bm_gemm_set_split(self._h, mode)
        if rc != BM_OK:
            raise BmGemmError(rc, "bm_gemm_set_split")

    def schedule(self) -> dict:
        si = ScheduleInfo()
        rc = self._lib.bm_gemm_query_schedule(self._h, ctypes.byref(si))
        if rc != BM_OK:
            raise BmGemmError(rc, "bm_gemm_query_schedule")
        return {f: getattr(si, f) for f, _ in ScheduleInfo._fields_}

    def status(self) -> tuple[int, int]:
        """(return code, device status bits); synchronises the device."""
        bits = ctypes.c_uint32(0)
        rc = self._lib.bm_gemm_status(self._h, ctypes.byref(bits))
        return rc, bits.value

    def set_debug(self, timeout_ns: int, flags: int) -> None:
        rc = self._lib.bm_gemm_set_debug(self._h, timeout_ns, flags)
        if rc != BM_OK:
            raise BmGemmError(rc, "bm_gemm_set_debug")

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.bm_gemm_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def fill(t, rows, cols, row_major, mode, seed=0, matrix_id=0, row0=0, full_ld=None, ld=None,
         stream=None) -> None:
    """bm_fill_fp16 into a CUDA tensor (modes 0, 1, 3, 4, 5)."""
    if ld is None:
        ld = cols if row_major else rows
    if full_ld is None:
        full_ld = ld
    rc = load().bm_fill_fp16(t.data_ptr(), rows, cols, ld, 1 if row_major else 0, row0, full_ld,
                             mode, seed, matrix_id, _stream_handle(stream))
    if rc != BM_OK:
        raise BmGemmError(rc, "bm_fill_fp16")


def alloc_operands(m, n, k, layout, device="cuda", mode=4, seed=0, row0=0, total_m=None):
    """Allocate and fill A, B and an empty C for `layout` on `device`.

    A is the row block [row0, row0 + m) of a logical total_m x k matrix (row-block
    sharding); B is the full n x k matrix. Values follow the counter-based
    generators (modes 0, 1, 3, 4, 5)."""
    import torch
    layout = layout.upper()
    total_m = total_m or m
    if layout == "NT":
        a = torch.empty((k, m), dtype=torch.float16, device=device)
        b = torch.empty((k, n), dtype=torch.float16, device=device)
        # A(m, k) at a[m + k*M] -> column-major logical storage (row_major=0)
        fill(a, m, k, row_major=False, mode=mode, seed=seed, matrix_id=0, row0=row0,
             full_ld=total_m, ld=m)
        fill(b, n, k, row_major=False, mode=mode, seed=seed, matrix_id=1)
    elif layout == "TN":
        a = torch.empty((m, k), dtype=torch.float16, device=device)
        b = torch.empty((n, k), dtype=torch.float16, device=device)
        fill(a, m, k, row_major=True, mode=mode, seed=seed, matrix_id=0, row0=row0, full_ld=k)
        fill(b, n, k, row_major=True, mode=mode, seed=seed, matrix_id=1)
    else:
        raise ValueError("layout must be NT or TN")
    c = torch.empty((n, m), dtype=torch.float16, device=device)
    return a, b, c


def run_noalloc(m, n, k, layout, a_ptr, b_ptr, c_ptr, lda=0, ldb=0, ldc=0, variant=0,
                stream=None, wait=True) -> tuple[int, int]:
    """bm_gemm_run_noalloc: one GEMM with no device allocation (the kernel's
    error word lives in the library's static device array). For callers that
    cannot call cudaMalloc. The first call on a device does the per-device
    set-up; calls that overlap on the GPU share the array and race on it.
    Returns (status code, device error bits); wait=False returns at once."""
    lib = load()
    fn = lib.bm_gemm_run_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.POINTER(GemmDesc), ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint32)]
    d = make_desc(m, n, k, layout, a_ptr, b_ptr, c_ptr, lda, ldb, ldc, variant)
    bits = ctypes.c_uint32(0)
    rc = fn(ctypes.byref(d), _stream_handle(stream), ctypes.byref(bits) if wait else None)
    return rc, bits.value
