"""build.sh / run.sh / summarize.py and the benchmark_host command line, on CPU.

Pattern of the reference's tests/test_run_device_compatibility.py: a fake
nvidia-smi and fake benchmark binaries on disk drive the runner end to end
without a GPU; the device gate must admit compute capability 10.0 only.
"""
from __future__ import annotations

import csv
import os
import shutil
import stat
import subprocess
import textwrap

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "best-matmul_b200")
BUILD = os.path.join(PKG, "build.sh")
RUN = os.path.join(PKG, "run.sh")
HEADER = ("id\tversion\tcta_m\tcta_n\tcta_k\tpipe\tgmma_n\tcompute_threads\tproducer_threads\t"
          "inflight\tepilogue\tbinary\tcta_group\tmma_per_k\tvariant\tstrict")


def _exe(path, body):
    with open(path, "w") as f:
        f.write(body)
    os.chmod(path, os.stat(path).st_mode | stat.S_IEXEC)


@pytest.fixture
def fake_env(tmp_path):
    """Fake nvidia-smi (capability from FAKE_CAP) and two fake binaries."""
    smi = tmp_path / "nvidia-smi"
    _exe(smi, textwrap.dedent("""\
        #!/usr/bin/env bash
        case "$*" in
          *compute_cap*) echo "${FAKE_CAP:-10.0}" ;;
          *name*) echo "NVIDIA B200" ;;
          *) echo "fake nvidia-smi $*" ;;
        esac
        """))
    build = tmp_path / "build"
    build.mkdir()
    rows = [HEADER]
    for ident, p50 in (("sm100_a", "0.100000"), ("sm100_b", "0.125000")):
        binary = build / ident
        _exe(binary, textwrap.dedent(f"""\
            #!/usr/bin/env bash
            echo "args: $*"
            echo "p50_ms={p50} ms"
            echo "p99_ms=0.130000 ms"
            echo "TFLOPS_p50=1234.5"
            echo "warmup_launches=300, warmup_stable=yes"
            echo "batch_drift_pct=0.5 % (last/first quarter medians)"
            """))
        _exe(str(binary) + ".validate", "#!/usr/bin/env bash\necho All full-output regressions PASS\n")
        rows.append("\t".join([ident, "sm100", "256", "512", "64", "4", "256", "256", "32", "1", "1",
                               str(binary), "2", "2", "5", "1"]))
    (build / "manifest.tsv").write_text("\n".join(rows) + "\n")
    env = dict(os.environ, NVIDIA_SMI=str(smi), NCU="false")
    return tmp_path, build, env


def _run(args, env, check=True):
    res = subprocess.run(["bash", RUN] + args, env=env, capture_output=True, text=True, timeout=120)
    if check and res.returncode != 0:
        raise AssertionError(res.stdout + res.stderr)
    return res


def test_build_dry_run_lists_every_variant_and_manifest_header():
    res = subprocess.run(["bash", BUILD, "--suite", "all", "--with-validation", "--dry-run"],
                         capture_output=True, text=True, timeout=60)
    assert res.returncode == 0, res.stderr
    out = res.stdout
    assert HEADER in out
    for v in range(0, 6):
        assert f"-DSM100_VARIANT={v}" in out
    assert "compute_100a" in out and "sm_100a" in out
    assert out.count("full_output_validation.cu") == out.count("benchmark_host.cu")


def test_build_rejects_bad_options():
    res = subprocess.run(["bash", BUILD, "--suite", "bogus"], capture_output=True, text=True)
    assert res.returncode == 2 and "--suite" in res.stderr


@pytest.mark.parametrize("mode,needle", [("nsys", "not installed"), ("sanitize", "closed on this pool"),
                                         ("disasm", "not provided"), ("bogus", "Unknown mode")])
def test_run_modes_not_offered(fake_env, mode, needle):
    _, build, env = fake_env
    res = _run(["--mode", mode, "--build-dir", str(build)], env, check=False)
    assert res.returncode != 0 and needle in res.stderr


def test_device_gate_rejects_hopper_and_admits_b200(fake_env):
    tmp, build, env = fake_env
    res = _run(["--mode", "check", "--build-dir", str(build), "--output-dir", str(tmp / "o1")],
               dict(env, FAKE_CAP="9.0"), check=False)
    assert res.returncode != 0 and "compute capability 9.0" in res.stderr
    res = _run(["--mode", "check", "--build-dir", str(build), "--output-dir", str(tmp / "o2"),
                "--timeout", "0"], dict(env, FAKE_CAP="10.0"))
    logs = sorted(p.name for p in (tmp / "o2").iterdir() if p.name.startswith("check_"))
    # K tiles {1, 2, S, S+1, 2S+1} with S = 4 -> 5 logs per id and layout
    assert len(logs) == 2 * 2 * 5
    assert "args: 512 1024 64 N T 3 event 1 1 2" in (tmp / "o2" / "check_sm100_a_NT_k1.log").read_text()


def test_bench_mode_writes_runs_and_summary(fake_env):
    tmp, build, env = fake_env
    out = tmp / "bench"
    _run(["--mode", "bench", "--build-dir", str(build), "--output-dir", str(out), "--repeats", "2",
          "--shapes", "4096x4096x4096", "--baseline", "sm100_a", "--timeout", "0"], env)
    with open(out / "summary.csv") as f:
        rows = {(r["id"], r["layout"]): r for r in csv.DictReader(f)}
    assert len(rows) == 4
    a = rows[("sm100_a", "NT")]
    assert float(a["median_p50_ms"]) == 0.1
    assert abs(float(a["tflops_from_median_p50"]) - 2 * 4096 ** 3 / (0.1 * 1e9)) < 1e-6
    assert abs(float(rows[("sm100_b", "TN")]["speedup_vs_baseline"]) - 0.8) < 1e-9
    with open(out / "runs.csv") as f:
        assert len(list(csv.DictReader(f))) == 8
    # the runner refuses to overwrite a result directory
    res = _run(["--mode", "bench", "--build-dir", str(build), "--output-dir", str(out)], env, check=False)
    assert res.returncode != 0 and "exists" in res.stderr


def test_validate_mode_writes_status_sidecars(fake_env):
    tmp, build, env = fake_env
    out = tmp / "val"
    _run(["--mode", "validate", "--build-dir", str(build), "--output-dir", str(out)], env)
    for ident in ("sm100_a", "sm100_b"):
        with open(out / f"validate_{ident}.status.tsv") as f:
            row = next(csv.DictReader(f, delimiter="\t"))
        assert row["status"] == "PASS" and row["exit_code"] == "0"


def test_validate_failure_is_recorded(fake_env):
    tmp, build, env = fake_env
    _exe(str(build / "sm100_b") + ".validate", "#!/usr/bin/env bash\necho mismatch >&2\nexit 3\n")
    out = tmp / "valfail"
    res = _run(["--mode", "validate", "--build-dir", str(build), "--output-dir", str(out)], env, check=False)
    assert res.returncode != 0
    with open(out / "validate_sm100_b.status.tsv") as f:
        assert next(csv.DictReader(f, delimiter="\t"))["status"] == "FAIL"


def test_manifest_tampering_is_rejected(fake_env):
    tmp, build, env = fake_env
    text = (build / "manifest.tsv").read_text().replace("\tsm100\t", "\tv3\t", 1)
    (build / "manifest.tsv").write_text(text)
    res = _run(["--mode", "check", "--build-dir", str(build), "--dry-run"], env, check=False)
    assert res.returncode != 0 and "version" in res.stderr


def test_shape_must_divide_strict_tiles(fake_env):
    _, build, env = fake_env
    res = _run(["--mode", "bench", "--build-dir", str(build), "--shapes", "4096x4096x4000",
                "--dry-run"], env, check=False)
    assert res.returncode != 0 and "not a multiple" in res.stderr


@pytest.fixture(scope="module")
def host_binary(tmp_path_factory):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    out = tmp_path_factory.mktemp("hb") / "benchmark_host"
    lib = os.path.join(PKG, "lib")
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O1", "-std=c++17",
           "-DSM100_VARIANT=5", os.path.join(PKG, "harness", "benchmark_host.cu"), "-o", str(out),
           f"-L{lib}", "-lbmgemm", "-Xlinker", "-rpath", "-Xlinker", lib]
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stderr
    return str(out)


def test_benchmark_host_help_and_argument_errors(host_binary):
    res = subprocess.run([host_binary, "--help"], capture_output=True, text=True)
    assert res.returncode == 0 and "sm100_tcgen05_2cta_256x512x64_s4" in res.stdout
    assert "Defaults: 4096 4096 4096 N T 2 event 20 20 200" in res.stdout
    cases = [
        (["4096", "4096", "4096", "N", "N"], "Only NT and TN"),
        (["4096", "4096", "4000", "N", "T"], "CTA_K == 0"),
        (["4096", "4096", "4096", "N", "T", "2", "event", "20x"], "Invalid integer for per_batch"),
        (["4096", "4096", "4096", "N", "T", "7"], "INPUT_MODE"),
        (["4096", "4096", "4096", "N", "T", "2", "clock"], "wall or event"),
        (["0", "4096", "4096"], "M,N,K > 0"),
        (["4096", "4096", "4096", "N", "T", "2", "event", "20", "20", "1"], "batches >= 2"),
        (["65536", "65536", "64", "N", "T"], "exceeds supported range"),
    ]
    for args, needle in cases:
        res = subprocess.run([host_binary] + args, capture_output=True, text=True)
        assert res.returncode != 0, args
        assert needle in res.stdout + res.stderr, (args, res.stdout, res.stderr)
