"""The C++ drop-in harness on a B200: native full-output regressions of every
built variant (run.sh --mode validate) and one short benchmark_host run whose
key=value lines follow the reference's output contract."""
from __future__ import annotations

import csv
import os
import re
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "best-matmul_b200")
BUILD_DIR = os.path.join(PKG, "build", "core")


@pytest.fixture(scope="module")
def manifest():
    import importlib.util
    spec = importlib.util.spec_from_file_location("bm_build", os.path.join(PKG, "build.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    path = mod.build_harness()
    with open(path) as f:
        return {r["id"]: r for r in csv.DictReader(f, delimiter="\t")}


def test_native_full_output_validation_all_variants(manifest, tmp_path):
    out = tmp_path / "validate"
    res = subprocess.run(["bash", os.path.join(PKG, "run.sh"), "--mode", "validate", "--build-dir",
                          BUILD_DIR, "--output-dir", str(out), "--timeout", "600"],
                         capture_output=True, text=True, timeout=1800)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    for ident in manifest:
        text = (out / f"validate_{ident}.log").read_text()
        assert "All full-output regressions PASS" in text, ident
        assert "Mapping PASS" in text, ident


@pytest.mark.parametrize("layout", ["NT", "TN"])
def test_benchmark_host_reports_contract_keys(manifest, layout):
    binary = manifest["sm100_auto"]["binary"]
    res = subprocess.run([binary, "4096", "4096", "4096", layout[0], layout[1], "4", "event", "10",
                          "20", "5"], capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-2000:]
    out = res.stdout
    for key in ("p50_ms", "p99_ms", "TFLOPS_p50", "warmup_launches", "warmup_stable",
                "batch_drift_pct"):
        assert re.search(r"\b" + key + r"=", out), key
    assert "Validation [precheck]: 16 sampled entries PASS" in out
    assert "Strict validation [postcheck]: 64 entries" in out
    tflops = float(re.search(r"TFLOPS_p50=([0-9.]+)", out).group(1))
    assert tflops > 500.0
