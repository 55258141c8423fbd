"""Row-block-sharded FP16 GEMM across the GPUs of one node.

    python -m torch.distributed.run --nproc-per-node P --master-addr 127.0.0.1 \\
        best-matmul_b200/sharded_gemm.py [--m 32768 --n 32768 --k 32768 --layout NT]
        [--reps 5] [--warmup 2] [--gather]

Each rank computes its row block of C = A * B^T with the sm_100a kernel (no
communication). Time = max over ranks of the per-rank CUDA-event time of
`reps` back-to-back launches; TFLOP/s counts the whole GEMM. With --gather the
NCCL all-gather of C plus the re-layout into the global column-major C is
timed separately (never part of the GEMM figure). Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from datetime import timedelta

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--m", type=int, default=32768)
    ap.add_argument("--n", type=int, default=32768)
    ap.add_argument("--k", type=int, default=32768)
    ap.add_argument("--layout", default="NT")
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--gather", action="store_true")
    ap.add_argument("--variant", type=int, default=0)
    args = ap.parse_args()

    import torch
    import torch.distributed as dist

    import sharder

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    sg = sharder.ShardedGemm(args.m, args.n, args.k, args.layout, rank, world,
                             variant=args.variant, device=dev)
    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        sg.launch(stream)
    torch.cuda.synchronize()
    if sg.gemm is not None:
        rc, bits = sg.gemm.status()
        if rc != 0:
            raise SystemExit(f"rank {rank}: kernel status {rc} bits {bits:#x}")
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.reps):
        sg.launch(stream)
    e1.record(stream)
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / args.reps], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    total_flops = 2.0 * args.m * args.n * args.k
    result = {
        "config": f"sharded FP16 GEMM {args.m}x{args.n}x{args.k} {args.layout}, row blocks over {world} GPU(s)",
        "world": world, "rows_per_rank": [b.rows for b in sg.blocks], "ms_per_gemm_max_over_ranks": ms,
        "tflops": total_flops / (ms * 1e-3) / 1e12,
        "kernel": sg.gemm.info()["name"] if sg.gemm is not None else None,
    }
    if args.gather and world > 1:
        out = torch.empty((args.n, args.m), dtype=torch.float16, device=dev)
        sg.gather(out=out)
        torch.cuda.synchronize()
        dist.barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        sg.gather(out=out)
        g1.record(stream)
        torch.cuda.synchronize()
        tg = torch.tensor([g0.elapsed_time(g1)], dtype=torch.float64, device=dev)
        dist.all_reduce(tg, op=dist.ReduceOp.MAX)
        nbytes = args.m * args.n * 2
        result["allgather_relayout_ms"] = float(tg.item())
        result["allgather_algbw_GBps"] = nbytes / (float(tg.item()) * 1e-3) / 1e9
    sg.close()
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
