"""Aggregate run.sh bench logs into runs.csv and summary.csv.

    python summarize.py RESULT_DIR BASELINE_ID

Only the plain timing logs listed in bench_index.tsv are read (never profiler
logs). Per (variant, shape, layout): the median over processes of each
process's p50 batch latency, TFLOP/s = 2MNK / that median, min/max p50, a
speed-up against BASELINE_ID on the same shape/layout, and how many runs were
flagged (warm-up not stable, or drift over 5 %). Same rules as the reference's
aggregation (scripts/common/runner_common.sh:439-484).
"""
from __future__ import annotations

import csv
import math
import pathlib
import re
import statistics
import sys

KEYS = ("p50_ms", "p99_ms", "TFLOPS_p50", "warmup_launches", "warmup_stable", "batch_drift_pct")


def parse_log(text: str, name: str) -> dict:
    row = {}
    for key in KEYS:
        m = re.search(r"\b" + key + r"=([^\s,]+)", text)
        if not m:
            raise SystemExit(f"missing {key} in {name}")
        row[key] = m.group(1)
    for key in ("p50_ms", "p99_ms", "TFLOPS_p50", "batch_drift_pct"):
        v = float(row[key])
        if not math.isfinite(v) or (key != "batch_drift_pct" and v <= 0):
            raise SystemExit(f"invalid {key} in {name}")
    return row


def main(root: pathlib.Path, baseline: str) -> None:
    configs = {}
    manifest = root / "manifest.tsv"
    if manifest.exists():
        with manifest.open() as f:
            configs = {r["id"]: r for r in csv.DictReader(f, delimiter="\t")}
    with (root / "bench_index.tsv").open() as f:
        index = list(csv.DictReader(f, delimiter="\t"))
    rows, groups = [], {}
    for entry in index:
        row = dict(entry)
        row.update(parse_log((root / entry["log"]).read_text(), entry["log"]))
        flags = []
        if row["warmup_stable"] != "yes":
            flags.append("warmup_not_stable")
        if abs(float(row["batch_drift_pct"])) > 5:
            flags.append("drift_over_5pct")
        row["warning"] = ";".join(flags)
        rows.append(row)
        groups.setdefault((row["id"], row["shape"], row["layout"]), []).append(row)
    if not rows:
        raise SystemExit("no bench runs")
    with (root / "runs.csv").open("w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=list(rows[0]))
        w.writeheader()
        w.writerows(rows)
    out = []
    for (ident, shape, layout), items in groups.items():
        p50s = [float(x["p50_ms"]) for x in items]
        med = statistics.median(p50s)
        m, n, k = map(int, shape.split("x"))
        ref = groups.get((baseline, shape, layout))
        speedup = statistics.median(float(x["p50_ms"]) for x in ref) / med if ref else ""
        cfg = configs.get(ident, {})
        out.append({
            "id": ident, "shape": shape, "layout": layout, "repeats": len(items),
            "cta": f"{cfg.get('cta_m', '?')}x{cfg.get('cta_n', '?')}x{cfg.get('cta_k', '?')}",
            "pipe": cfg.get("pipe", ""), "cta_group": cfg.get("cta_group", ""),
            "median_p50_ms": med, "min_p50_ms": min(p50s), "max_p50_ms": max(p50s),
            "tflops_from_median_p50": 2 * m * n * k / (med * 1e9), "baseline": baseline,
            "speedup_vs_baseline": speedup,
            "flagged_runs": sum(bool(x["warning"]) for x in items),
        })
    with (root / "summary.csv").open("w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=list(out[0]))
        w.writeheader()
        w.writerows(out)
    print(f"Saved {len(rows)} runs and {len(out)} groups to {root}")


if __name__ == "__main__":
    if len(sys.argv) != 3:
        raise SystemExit("usage: summarize.py RESULT_DIR BASELINE_ID")
    main(pathlib.Path(sys.argv[1]), sys.argv[2])
