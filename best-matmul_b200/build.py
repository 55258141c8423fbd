"""Build the sm_100a GEMM library (lib/libbmgemm.so) and the C++ harness.

    python best-matmul_b200/build.py [--force] [--verbose]

nvcc cross-compiles for sm_100a without a GPU. The library links the CUDA
runtime statically so it does not depend on which libcudart a host process
(e.g. PyTorch) loaded first.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB_DIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIB_DIR, "libbmgemm.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xptxas", "-v",
                     "-Xcompiler", "-fPIC", "-cudart", "static"]


def nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def _sources():
    return [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC))
            if f.endswith((".cu", ".cuh"))] + [os.path.join(ROOT, "include", "bm_gemm.h")]


def _stale(target, sources) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def build_library(force=False, verbose=False) -> str:
    os.makedirs(LIB_DIR, exist_ok=True)
    if not force and not _stale(LIB, _sources()):
        return LIB
    cmd = [nvcc()] + NVCC_FLAGS + ["-shared", "-o", LIB, os.path.join(CSRC, "bm_gemm.cu")]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or res.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed building {LIB}")
    with open(os.path.join(LIB_DIR, "ptxas_info.txt"), "w") as f:
        f.write(" ".join(cmd) + "\n" + res.stderr)
    return LIB


HARNESS_DIR = os.path.join(HERE, "build", "core")
HARNESS_SOURCES = [os.path.join(HERE, "harness", f) for f in ("benchmark_host.cu", "full_output_validation.cu")]


def build_harness(force=False, verbose=False) -> str:
    """benchmark_host + full_output_validation per variant, via build.sh (manifest.tsv)."""
    manifest = os.path.join(HARNESS_DIR, "manifest.tsv")
    deps = _sources() + HARNESS_SOURCES + [
        os.path.join(HERE, "kernels", "sm100_fp16_gemm.cuh"), os.path.join(HERE, "build.sh")] + [
        os.path.join(HERE, "host", f) for f in os.listdir(os.path.join(HERE, "host"))]
    if not force and not _stale(manifest, deps):
        return manifest
    res = subprocess.run(["bash", os.path.join(HERE, "build.sh"), "--suite", "core",
                          "--with-validation"], capture_output=True, text=True)
    if verbose or res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
    if res.returncode != 0:
        raise RuntimeError("build.sh failed")
    return manifest


STATS_LIB = os.path.join(LIB_DIR, "libbmgemm_stats.so")


def build_stats_library(force=False, verbose=False) -> str:
    """Diagnostics build (-DBM_KERNEL_STATS): the same kernels with per-CTA
    pipeline counters and per-tile timestamps (harness/pipeline_timeline.py)."""
    os.makedirs(LIB_DIR, exist_ok=True)
    if not force and not _stale(STATS_LIB, _sources()):
        return STATS_LIB
    cmd = [nvcc()] + NVCC_FLAGS + ["-DBM_KERNEL_STATS", "-shared", "-o", STATS_LIB,
                                   os.path.join(CSRC, "bm_gemm.cu")]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or res.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed building {STATS_LIB}")
    return STATS_LIB


def build_all(force=False, verbose=False) -> None:
    build_library(force, verbose)
    build_harness(force, verbose)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--stats", action="store_true",
                    help="also build lib/libbmgemm_stats.so (pipeline counters, diagnostics only)")
    ap.add_argument("--lib-only", action="store_true",
                    help="build only lib/libbmgemm.so (build.sh calls this before the harness)")
    args = ap.parse_args()
    if args.lib_only:
        build_library(args.force, args.verbose)
    else:
        build_all(args.force, args.verbose)
    if args.stats:
        build_stats_library(args.force, args.verbose)
    print("built", LIB)
