"""Benchmark of the sm_100a FP16 GEMM hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: FP16 GEMM 4096^3, NT and TN, uniform[-1,1]
inputs, FP32 accumulation, FP16 C. One step is one measurement batch of the
reference harness (per_batch = 20 launches, host/common.cuh:80): 10 NT and 10
TN GEMMs, alternating. Under torchrun each rank owns a 4096-row block of a
(N*4096) x 4096 x 4096 GEMM with B replicated (row-block sharding, no
collective in the timed region): weak scaling.

Inputs rotate over enough buffer sets that every launch reads operands last
touched more than 3x L2 (126 MB) earlier, so no launch starts with warm L2.

--impl reference times the reference's own CPU GEMM (reference_gemm_entry of
host/validation.cuh, compiled from the reference sources into oracle/_ref) on
this host's cores over a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "best-matmul_b200")
ORACLE_DIR = os.path.join(ROOT, "oracle")
sys.path.insert(0, PKG)

METRIC = "FP16 GEMM TFLOP/s (4096^3 NT+TN, FP32 accumulate) per job"
SIZE = 4096
LAUNCHES_PER_STEP = 20
L2_BYTES = 126 * 1024 * 1024


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--size", type=int, default=SIZE, help="M (per rank) = N = K")
    ap.add_argument("--variant", type=int, default=0)
    ap.add_argument("--split", choices=["none", "auto"], default="auto",
                    help="schedule of leftover tiles (bm_gemm_set_split)")
    ap.add_argument("--no-cublas", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    return ap.parse_args()


def measured_peaks():
    """(burst TFLOP/s, sustained TFLOP/s, HBM GB/s, source) for dense bf16/fp16."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return (float(p["bf16_tflops"]), float(p.get("bf16_tflops_sustained", p["bf16_tflops"])),
                float(p["hbm_gbs"]), "measured")
    except Exception:
        return 1590.0, 1400.0, 6650.0, "fallback"


def profiled_traffic(size):
    """DRAM bytes per launch from the committed ncu summary (None if absent)."""
    path = os.path.join(ROOT, "profiles", f"gemm_{size}_dram_traffic.txt")
    try:
        vals = {}
        with open(path) as f:
            for line in f:
                parts = line.split()
                if len(parts) >= 2 and parts[0] in ("NT", "TN"):
                    vals[parts[0]] = float(parts[1])
        if vals:
            return vals
    except OSError:
        pass
    return None


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, period_s: float = 0.01):
        self.samples, self.reasons, self.ok = [], 0, False
        self._stop = threading.Event()
        self._period = period_s
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            # NVML and CUDA may number devices differently: match on PCI location.
            props = torch.cuda.get_device_properties(device_index)
            want = (int(props.pci_domain_id), int(props.pci_bus_id), int(props.pci_device_id))
            self._h = None
            for i in range(pynvml.nvmlDeviceGetCount()):
                h = pynvml.nvmlDeviceGetHandleByIndex(i)
                pi = pynvml.nvmlDeviceGetPciInfo(h)
                if (int(pi.domain), int(pi.bus), int(pi.device)) == want:
                    self._h = h
                    break
            if self._h is None:
                raise RuntimeError(f"no NVML device at PCI {want}")
            self._nvml = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # NVML missing: report, do not fail the bench
            self.error = str(e)

    def _run(self):
        n = self._nvml
        while not self._stop.is_set():
            try:
                self.samples.append(n.nvmlDeviceGetClockInfo(self._h, n.NVML_CLOCK_SM))
                self.reasons |= n.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            except Exception:
                pass
            time.sleep(self._period)

    def __enter__(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self.ok:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml_unavailable"]}
        names = [v for k, v in self.REASONS.items() if self.reasons & k and k != 0x1]
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(self.samples)}


# ------------------------------------------------------------------ CPU arm
def cpu_reference_sample(size, seconds, layouts=("NT", "TN")):
    """Time the reference's reference_gemm_entry (oracle/_ref) - or, where the
    reference could not be compiled, the C oracle port - on all host threads
    over a bounded sample of the workload's output entries."""
    import numpy as np
    sys.path.insert(0, ORACLE_DIR)
    from oracle import REF_LIB, Oracle, RefLib, default_threads

    threads = default_threads()
    orc = Oracle()
    kind = "reference" if os.path.exists(REF_LIB) else "port"
    ref = RefLib() if kind == "reference" else None
    m = n = k = size
    results = {}
    total_flops = total_time = 0.0
    entries_done = 0
    for layout in layouts:
        a, b = orc.make_inputs(m, n, k, layout, 4, seed=0)
        lda, ldb = (m, n) if layout == "NT" else (k, k)
        prob = ref.problem(m, n, k, layout, a=a, b=b) if ref else None

        def run(rows, cols):
            if prob is not None:
                return prob.entries(rows, cols, threads)
            return orc.entries_f64(k, layout, a, lda, b, ldb, rows, cols, threads)

        # calibrate on a small block, then size the sample to the time budget
        rng = np.random.default_rng(0)
        cal = max(threads * 4, 64)
        rows, cols = rng.integers(0, m, cal), rng.integers(0, n, cal)
        t0 = time.perf_counter()
        run(rows, cols)
        per_entry = (time.perf_counter() - t0) / cal
        count = int(max(cal, min(m * n, (seconds / len(layouts)) / max(per_entry, 1e-9))))
        # a contiguous block of whole columns (what a CPU harness would compute)
        cols_n = max(1, count // m)
        cc = np.repeat(np.arange(cols_n) % n, m)
        rr = np.tile(np.arange(m), cols_n)
        t0 = time.perf_counter()
        run(rr, cc)
        dt = time.perf_counter() - t0
        flops = 2.0 * k * rr.size
        results[layout] = {"entries": int(rr.size), "seconds": dt, "tflops": flops / dt / 1e12}
        total_flops += flops
        total_time += dt
        entries_done += rr.size
        if prob is not None:
            prob.close()
    value = total_flops / total_time / 1e12
    sample = (f"{entries_done} output entries ({', '.join(f'{l}: {r['entries']}' for l, r in results.items())}) "
              f"of the {size}^3 GEMMs = whole columns of C, FP64 accumulate, {threads} threads")
    return {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": kind, "sample": sample,
            "per_layout_tflops": {l: r["tflops"] for l, r in results.items()}}


def run_reference_arm(args, rank, world):
    if rank != 0:
        return
    per_step_seconds = max(0.5, min(args.cpu_seconds, 120.0 / max(1, args.steps + args.warmup)))
    for _ in range(args.warmup):
        cpu_reference_sample(args.size, per_step_seconds / 4)
    vals = []
    t_all = time.perf_counter()
    for _ in range(args.steps):
        vals.append(cpu_reference_sample(args.size, per_step_seconds))
    elapsed = time.perf_counter() - t_all
    value = statistics.median(v["value"] for v in vals)
    cb = dict(vals[-1])
    cb["value"] = value
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": elapsed * 1000.0 / max(1, args.steps), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
        "config": {"workload": f"FP16 GEMM {args.size}^3 NT+TN, uniform[-1,1] seed 0",
                   "m": args.size, "n": args.size, "k": args.size, "layouts": ["NT", "TN"],
                   "parallelism": "host threads (rank 0 only)"},
        "cpu_baseline": cb,
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU arm
def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        return run_reference_arm(args, rank, world)

    import torch
    import torch.distributed as dist
    import bmgemm as bm

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
    m = n = k = args.size
    flops = 2.0 * m * n * k
    set_bytes = 2 * (m * k + n * k + m * n) * 2  # NT + TN operand sets
    n_sets = max(2, -(-3 * L2_BYTES // set_bytes) + 1)
    sets = []
    for s in range(n_sets):
        entry = {}
        for layout in ("NT", "TN"):
            a, b, c = bm.alloc_operands(m, n, k, layout, device=dev, mode=4, seed=s,
                                        row0=rank * m, total_m=world * m)
            g = bm.Gemm.from_tensors(a, b, c, layout, variant=args.variant)
            g.set_split(bm.SPLIT_NONE if args.split == "none" else bm.SPLIT_AUTO)
            entry[layout] = (a, b, c, g)
        sets.append(entry)
    info = {l: sets[0][l][3].info() for l in ("NT", "TN")}
    sched = sets[0]["NT"][3].schedule()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)

    order = [("NT" if i % 2 == 0 else "TN", (i // 2)) for i in range(LAUNCHES_PER_STEP)]

    def step(step_idx, events=None):
        for i, (layout, j) in enumerate(order):
            g = sets[(step_idx * (LAUNCHES_PER_STEP // 2) + j) % n_sets][layout][3]
            if events is not None:
                events[i][0].record(stream)
            g.launch(stream)
            if events is not None:
                events[i][1].record(stream)

    # warm-up (untimed)
    for w in range(max(3, args.warmup)):
        step(w)
    torch.cuda.synchronize()
    for entry in sets:
        for layout in ("NT", "TN"):
            rc, bits = entry[layout][3].status()
            if rc != bm.BM_OK:
                raise SystemExit(f"GEMM status {rc} bits {bits:#x} during warm-up")

    # timed region: K steps, per-launch events for the kernel roofline
    ev = [[[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)]
           for _ in range(LAUNCHES_PER_STEP)] for _ in range(args.steps)]
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        barrier()
        torch.cuda.synchronize()
        t_start.record(stream)
        for s_i in range(args.steps):
            step(s_i, ev[s_i])
        t_end.record(stream)
        torch.cuda.synchronize()
        barrier()
    elapsed_ms = t_start.elapsed_time(t_end)
    per_launch = {"NT": [], "TN": []}
    for s_i in range(args.steps):
        for i, (layout, _) in enumerate(order):
            per_launch[layout].append(ev[s_i][i][0].elapsed_time(ev[s_i][i][1]))
    for entry in sets:
        for layout in ("NT", "TN"):
            rc, bits = entry[layout][3].status()
            if rc != bm.BM_OK:
                raise SystemExit(f"GEMM status {rc} bits {bits:#x} in the timed region")

    t_max = torch.tensor([elapsed_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
    elapsed_max = float(t_max.item())
    total_flops = flops * LAUNCHES_PER_STEP * args.steps * world
    value = total_flops / (elapsed_max * 1e-3) / 1e12

    # kernel roofline: algorithmic FLOPs per launch / mean CUDA-event duration.
    # The timed loop runs back to back for a long stretch under the 1 kW power
    # cap, so the matching denominator is the sustained dense-GEMM peak; the
    # burst figure is reported beside it.
    peak_burst, peak_sust, hbm_peak, peak_kind = measured_peaks()
    mean_ms = {l: statistics.mean(v) for l, v in per_launch.items()}
    med_ms = {l: statistics.median(v) for l, v in per_launch.items()}
    launch_ms = statistics.mean(per_launch["NT"] + per_launch["TN"])
    achieved = flops / (launch_ms * 1e-3) / 1e12
    traffic = profiled_traffic(args.size)
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak_sust, "unit": "TFLOP/s",
                "frac": achieved / peak_sust,
                "peak_source": f"{peak_kind} dense bf16/fp16 GEMM, sustained (timed loop is "
                               f"{elapsed_max / 1e3:.2f} s back to back)",
                "peak_burst": peak_burst, "frac_of_burst": achieved / peak_burst,
                "traffic": (statistics.mean(traffic.values()) if traffic else None),
                "traffic_source": "profiles/gemm_%d_dram_traffic.txt (ncu dram bytes/launch)" % args.size,
                "algorithmic_bytes": 2.0 * (m * k + n * k + m * n),
                "per_layout_tflops": {l: flops / (mean_ms[l] * 1e-3) / 1e12 for l in mean_ms},
                "per_layout_median_ms": med_ms}

    # cuBLAS (torch.matmul, FP32 accumulate) on the same shapes, buffers and
    # rotation. Batches of ours and of cuBLAS alternate, so both run in the
    # same power/thermal state; per-launch CUDA events on the same stream.
    cublas = None
    if not args.no_cublas:
        def cublas_one(entry, layout):
            a, b, c, _ = entry[layout]
            if layout == "NT":
                torch.matmul(b.t(), a, out=c)  # (N,K)@(K,M) -> c[n][m]
            else:
                torch.matmul(b, a.t(), out=c)

        def cublas_batch(step_idx, events=None):
            for i, (layout, j) in enumerate(order):
                if events is not None:
                    events[i][0].record(stream)
                cublas_one(sets[(step_idx * (LAUNCHES_PER_STEP // 2) + j) % n_sets], layout)
                if events is not None:
                    events[i][1].record(stream)

        for w in range(3):
            cublas_batch(w)
        torch.cuda.synchronize()
        rounds = max(5, min(args.steps, 40))
        ev_ours = [[[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in order]
                   for _ in range(rounds)]
        ev_cub = [[[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in order]
                  for _ in range(rounds)]
        for r in range(rounds):
            step(r, ev_ours[r])
            cublas_batch(r, ev_cub[r])
        torch.cuda.synchronize()
        pair = {"ours": {"NT": [], "TN": []}, "cublas": {"NT": [], "TN": []}}
        for r in range(rounds):
            for i, (layout, _) in enumerate(order):
                pair["ours"][layout].append(ev_ours[r][i][0].elapsed_time(ev_ours[r][i][1]))
                pair["cublas"][layout].append(ev_cub[r][i][0].elapsed_time(ev_cub[r][i][1]))
        tf = {who: {l: flops / (statistics.median(v) * 1e-3) / 1e12 for l, v in d.items()}
              for who, d in pair.items()}
        cublas = {"NT": tf["cublas"]["NT"], "TN": tf["cublas"]["TN"], "unit": "TFLOP/s",
                  "ours_interleaved": tf["ours"],
                  "ours_over_cublas": {l: tf["ours"][l] / tf["cublas"][l] for l in ("NT", "TN")},
                  "rounds": rounds,
                  "what": "torch.matmul fp16 (cuBLAS, FP32 accumulate), same buffers; batches of "
                          "20 launches alternating with ours; median per-launch event time"}

    # end to end through the C ABI with host buffers: per launch, H2D of A and
    # B from pinned memory, the GEMM, D2H of C, all on one stream.
    e2e = None
    if not args.no_e2e:
        host = {}
        for layout in ("NT", "TN"):
            a, b, c, _ = sets[0][layout]
            host[layout] = (a.cpu().pin_memory(), b.cpu().pin_memory(),
                            torch.empty(c.shape, dtype=c.dtype).pin_memory())
        e2e_steps = max(2, min(args.steps, 10))

        def e2e_step():
            for i, (layout, _) in enumerate(order):
                a, b, c, g = sets[i % 2][layout]
                ha, hb, hc = host[layout]
                a.copy_(ha, non_blocking=True)
                b.copy_(hb, non_blocking=True)
                g.launch(stream)
                hc.copy_(c, non_blocking=True)

        e2e_step()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        t = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_val = flops * LAUNCHES_PER_STEP * e2e_steps * world / (float(t.item()) * 1e-3) / 1e12
        e2e = {"value": e2e_val, "unit": "TFLOP/s",
               "h2d_bytes_per_step": LAUNCHES_PER_STEP * 2 * (m * k + n * k),
               "d2h_bytes_per_step": LAUNCHES_PER_STEP * 2 * m * n, "steps": e2e_steps}

    # optional all-gather of C over NVLink, timed separately (not in `value`)
    allgather = None
    if world > 1:
        c_local = sets[0]["NT"][2].reshape(-1)
        out = torch.empty(c_local.numel() * world, dtype=c_local.dtype, device=dev)
        for _ in range(3):
            dist.all_gather_into_tensor(out, c_local)
        torch.cuda.synchronize()
        a0 = torch.cuda.Event(enable_timing=True)
        a1 = torch.cuda.Event(enable_timing=True)
        reps = 10
        barrier()
        a0.record(stream)
        for _ in range(reps):
            dist.all_gather_into_tensor(out, c_local)
        a1.record(stream)
        torch.cuda.synchronize()
        tt = torch.tensor([a0.elapsed_time(a1) / reps], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        nbytes = out.numel() * out.element_size()
        allgather = {"ms": float(tt.item()), "bytes": nbytes,
                     "busbw_GBps": nbytes * (world - 1) / world / (float(tt.item()) * 1e-3) / 1e9}

    cpu_baseline = None
    if rank == 0 and world == 1:
        cpu_baseline = cpu_reference_sample(args.size, args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": elapsed_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
            "config": {
                "workload": f"FP16 GEMM {m}^3 per rank, NT and TN alternating, "
                            f"uniform[-1,1] FP16, FP32 accumulate, FP16 C",
                "m_per_rank": m, "n": n, "k": k, "global_m": m * world,
                "launches_per_step": LAUNCHES_PER_STEP,
                "parallelism": f"row-block dp{world} (A, C split by rows, B replicated)",
                "l2": f"{n_sets} rotating operand sets ({set_bytes * n_sets / 2**20:.0f} MiB) "
                      "> 3x L2 between reuses",
                "kernels": {l: info[l]["name"] for l in info},
                "grid": {l: info[l]["grid"][0] for l in info},
                "schedule": dict(sched, split=args.split),
            },
            "roofline": roofline, "cpu_baseline": cpu_baseline, "e2e": e2e,
            "gpu_launches": LAUNCHES_PER_STEP * args.steps, "clocks": clocks.summary(),
            "cublas": cublas, "allgather": allgather,
        }
        print(json.dumps(line), flush=True)

    for entry in sets:
        for layout in ("NT", "TN"):
            entry[layout][3].close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
