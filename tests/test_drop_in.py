"""Source-level drop-in: the reference's own benchmark_host.cu (unmodified,
compiled where it lies) builds against this repository's GEMM_KERNEL_HEADER
and reports the sm_100a backend. Needs the reference sources and a CUTLASS
include tree (for the reference's host headers); skipped where absent."""
from __future__ import annotations

import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "best-matmul_b200")
REF = os.environ.get("BM_REFERENCE_ROOT", "/root/reference")


def _cutlass_include():
    try:
        import flashinfer
    except Exception:
        return None
    path = os.path.join(os.path.dirname(flashinfer.__file__), "data", "cutlass", "include")
    return path if os.path.exists(os.path.join(path, "cutlass", "half.h")) else None


def test_reference_benchmark_host_compiles_against_sm100_backend(tmp_path):
    src = os.path.join(REF, "benchmark_host.cu")
    cut = _cutlass_include()
    if not os.path.exists(src) or cut is None:
        pytest.skip("reference sources or CUTLASS headers not present")
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    out = tmp_path / "ref_benchmark_host_sm100"
    header = os.path.join(PKG, "kernels", "sm100_fp16_gemm.cuh")
    lib = os.path.join(PKG, "lib")
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O1", "-std=c++17",
           "--expt-relaxed-constexpr", f"-I{REF}", f"-I{cut}",
           # the reference guards its runner with this macro (benchmark_host.cu:14,
           # :82); defining it compiles the with_prepared() call path
           "-DCUTLASS_ARCH_MMA_SM90_SUPPORTED", f'-DGEMM_KERNEL_HEADER="{header}"',
           "-DSM100_VARIANT=5", src, "-o", str(out), f"-L{lib}", "-lbmgemm",
           "-Xlinker", "-rpath", "-Xlinker", lib]
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-4000:]
    res = subprocess.run([str(out), "--help"], capture_output=True, text=True, timeout=60)
    assert res.returncode == 0
    assert "Kernel: sm100_tcgen05_2cta_256x512x64_s4" in res.stdout
    assert "tcgen05.mma kind::f16" in res.stdout
