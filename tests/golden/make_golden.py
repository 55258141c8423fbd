"""Generate tests/golden/reference_golden.json from the REFERENCE's own code.

    make -C oracle all ref && python tests/golden/make_golden.py

The values come from ggbond-x/best-matmul's host/common.cuh (GemmBuffers input
order, make_input_value, GemmProblem index functions) and host/validation.cuh
(reference_gemm_entry), compiled unmodified into oracle/_ref/libbm_ref.so. The
committed JSON lets tests pin the C oracle on machines where the reference
sources are absent (e.g. the GPU box).

Modes 4/5 (uniform / normal, not part of the reference) are recorded from the
C oracle itself as regression vectors for the device generator.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

from oracle import Oracle, RefLib  # noqa: E402

SHAPES = [(64, 48, 40), (256, 256, 192), (128, 96, 1000)]


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def grid_samples(m, n):
    rows = [int((m - 1) * r // 3) for r in range(4)]
    cols = [int((n - 1) * c // 3) for c in range(4)]
    rr = [r for r in rows for _ in cols]
    cc = [c for _ in rows for c in cols]
    rng = np.random.default_rng(12345)
    rr += rng.integers(0, m, 16).tolist()
    cc += rng.integers(0, n, 16).tolist()
    return rr, cc


def main() -> None:
    ref = RefLib()
    orc = Oracle()
    out = {"source": "reference host/common.cuh + host/validation.cuh compiled in place",
           "reference_cases": [], "generator_cases": []}
    for (m, n, k) in SHAPES:
        for layout in ("NT", "TN"):
            for mode in (0, 1, 2, 3):
                p = ref.problem(m, n, k, layout, mode=mode)
                a, b = p.export()
                rows, cols = grid_samples(m, n)
                vals = p.entries(rows, cols, threads=1).tolist()
                idx = {
                    "a": [p.index("a", r, q) for r, q in ((0, 0), (m - 1, 0), (0, k - 1), (m // 2, k // 3))],
                    "b": [p.index("b", c, q) for c, q in ((0, 0), (n - 1, 0), (0, k - 1), (n // 2, k // 3))],
                    "c": [p.index("c", r, c) for r, c in ((0, 0), (m - 1, 0), (0, n - 1), (m // 2, n // 3))],
                }
                case = {"m": m, "n": n, "k": k, "layout": layout, "mode": mode,
                        "sha_a": sha(a), "sha_b": sha(b), "a_head": a[:8].tolist(),
                        "b_head": b[:8].tolist(), "rows": rows, "cols": cols,
                        "entries": vals, "index": idx}
                if m * n <= 64 * 48:
                    full_r = np.repeat(np.arange(m), n)
                    full_c = np.tile(np.arange(n), m)
                    full = p.entries(full_r, full_c, threads=1)
                    case["full_sha_f64"] = sha(full.astype(np.float64))
                    case["full_sum"] = float(full.sum())
                out["reference_cases"].append(case)
                p.close()
    for (m, n, k) in SHAPES[:2]:
        for layout in ("NT", "TN"):
            for mode in (4, 5):
                a, b = orc.make_inputs(m, n, k, layout, mode, seed=0)
                out["generator_cases"].append({"m": m, "n": n, "k": k, "layout": layout,
                                               "mode": mode, "seed": 0, "sha_a": sha(a),
                                               "sha_b": sha(b), "a_head": a[:8].tolist(),
                                               "b_head": b[:8].tolist()})
    path = os.path.join(HERE, "reference_golden.json")
    with open(path, "w") as f:
        json.dump(out, f, indent=1)
    print("wrote", path, len(out["reference_cases"]), "reference cases")


if __name__ == "__main__":
    main()
