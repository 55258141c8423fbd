"""Per-tile pipeline timeline of one GEMM launch (diagnostics).

    python best-matmul_b200/build.py --lib-only --stats
    python best-matmul_b200/harness/pipeline_timeline.py [--size 4096 | --m M --n N --k K]
           [--layout TN] [--variant 0] [--split auto|none] [--reps 5]

Loads lib/libbmgemm_stats.so (the kernels built with -DBM_KERNEL_STATS), which
writes, per CTA, %globaltimer stamps of set-up, of every tile's MMA start and
end, of the epilogue's start, TMEM release and last store, plus the MMA
thread's clock64 cycles and data-wait cycles per tile. Prints, per tile index,
the means over the cluster leaders, and the MMA-thread cycles against the
tensor-pipe ideal of a whole tile: per 64-deep k-block, (tile rows per CTA x
tile columns x 64) multiply-adds at 4096 per cycle per SM (1024 cycles for the
256x512 pair tile). The stats build is for diagnosis only; its absolute times
include its own bookkeeping.
"""
from __future__ import annotations

import argparse
import ctypes
import os
import statistics
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
sys.path.insert(0, PKG)

# slot layout of StatSlot in csrc/gemm_sm100.cuh
T_ENTRY, T_EXIT, MMA_FIRST = 12, 13, 14
UNIT0, UNITS, UNIT_FIELDS = 16, 6, 7
UNIT_COUNT = UNIT0 + UNIT_FIELDS * UNITS
SETUP_ALLOC, SETUP_SYNC, SETUP_CLUSTER = UNIT_COUNT + 1, UNIT_COUNT + 2, UNIT_COUNT + 3
NUM_STATS = SETUP_CLUSTER + 1


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--size", type=int, default=4096)
    ap.add_argument("--m", type=int, default=0)
    ap.add_argument("--n", type=int, default=0)
    ap.add_argument("--k", type=int, default=0)
    ap.add_argument("--layout", default="TN")
    ap.add_argument("--variant", type=int, default=0)
    ap.add_argument("--split", choices=["auto", "none"], default="auto")
    ap.add_argument("--reps", type=int, default=5)
    args = ap.parse_args()

    import bmgemm as bm
    bm.LIB_PATH = os.path.join(PKG, "lib", "libbmgemm_stats.so")
    import torch
    lib = bm.load()
    lib.bm_gemm_debug_attach_stats.restype = ctypes.c_int
    lib.bm_gemm_debug_attach_stats.argtypes = [ctypes.c_void_p, ctypes.c_void_p]

    m, n, k = (args.m or args.size), (args.n or args.size), (args.k or args.size)
    a, b, c = bm.alloc_operands(m, n, k, args.layout, mode=4, seed=0)
    g = bm.Gemm.from_tensors(a, b, c, args.layout, variant=args.variant)
    g.set_split(bm.SPLIT_AUTO if args.split == "auto" else bm.SPLIT_NONE)
    info = g.info()
    grid, cg = info["grid"][0], info["cta_group"]
    st = torch.zeros(grid * NUM_STATS, dtype=torch.int64, device="cuda")
    if lib.bm_gemm_debug_attach_stats(g._h, ctypes.c_void_p(st.data_ptr())) != 0:
        raise SystemExit("attach failed")
    flush = torch.empty(256 * 2**20, dtype=torch.uint8, device="cuda")  # > L2 between launches
    durs = []
    for r in range(args.reps):
        flush.fill_(r)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.launch()
        e1.record()
        torch.cuda.synchronize()
        durs.append(e0.elapsed_time(e1) * 1e3)
    rc, bits = g.status()
    if rc != bm.BM_OK:
        raise SystemExit(f"kernel status {rc} bits {bits:#x}")
    s = st.view(grid, NUM_STATS).cpu().numpy().astype(float)
    t0 = s[:, T_ENTRY].min()
    us = lambda v: v / 1e3
    print(f"{m}x{n}x{k} {args.layout} {info['name']} grid={grid} schedule={g.schedule()}")
    print(f"event time per launch (us): {[round(d, 1) for d in durs]}")
    print(f"kernel span (first entry to last exit) {us(s[:, T_EXIT].max() - t0):.1f} us")
    lead = s[::cg]
    print("set-up (us after first entry, mean): TMEM allocated "
          f"{us((lead[:, SETUP_ALLOC] - t0).mean()):.2f}, CTA barrier {us((lead[:, SETUP_SYNC] - t0).mean()):.2f}, "
          f"cluster barrier {us((lead[:, SETUP_CLUSTER] - t0).mean()):.2f}, first MMA {us((lead[:, MMA_FIRST] - t0).mean()):.2f}")
    kb = (k + 63) // 64
    tile_m, tile_n = info["tile"][0], info["tile"][1]
    ideal_kb = (tile_m // cg) * tile_n * 64 // 4096  # MMA cycles per k-block per SM
    for u in range(UNITS):
        sel = lead[lead[:, UNIT_COUNT] > u]
        if len(sel) == 0:
            break
        base = UNIT0 + UNIT_FIELDS * u
        ms, me, es, er, ee = (sel[:, base + i] - t0 for i in range(5))
        wait, cyc = sel[:, base + 5], sel[:, base + 6]
        print(f"tile {u}: {len(sel)} pairs | MMA {us(ms.mean()):.1f} -> {us(me.mean()):.1f} us | "
              f"MMA-thread cycles {cyc.mean():.0f} (whole-tile ideal {kb * ideal_kb}: "
              f"{kb * ideal_kb / cyc.mean():.3f}), data waits {wait.mean():.0f} | accumulator ready "
              f"+{us((es - me).mean()):.1f} us, TMEM held {us((er - es).mean()):.2f} us, stores issued "
              f"+{us((ee - er).mean()):.2f} us | last store {us(ee.max()):.1f} us")
    g.close()


if __name__ == "__main__":
    main()
