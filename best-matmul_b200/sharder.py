"""Row-block sharding of one FP16 GEMM across the ranks of a process group.

The reference runs on one device only; this is the multi-GPU layer of the
B200 build. C(M,N) = A(M,K) * B(N,K)^T is split by rows: rank p owns the row
block [row0_p, row0_p + rows_p) of A and of C and holds all of B. Every rank
runs the same single-GPU kernel on its block with no communication; the
result stays distributed. gather_c() optionally assembles the global
column-major C on every rank: an all-gather of the per-rank blocks (NCCL over
NVLink on GPUs, gloo on CPU) followed by a strided copy that places each
block's rows into C (column-major C makes a row block strided, so the
gathered [P][N][rows] blocks are re-laid out to [N][M]).

Block sizes are multiples of `align` rows (the kernel's pair-tile height, and
a multiple of 8 so that NT leading dimensions stay 16-byte aligned); only the
last block may be shorter. Inputs come from the counter-based generators, so
every rank produces exactly its rows of the one global matrix.
"""
from __future__ import annotations

from dataclasses import dataclass

DEFAULT_ALIGN = 256


@dataclass(frozen=True)
class RowBlock:
    rank: int
    world: int
    row0: int
    rows: int
    m: int  # global M


def row_blocks(m: int, world: int, align: int = DEFAULT_ALIGN) -> list[RowBlock]:
    """Contiguous row blocks, sizes multiples of `align` (last may be short)."""
    if m <= 0 or world <= 0 or align <= 0 or align % 8:
        raise ValueError("need m > 0, world > 0 and align a positive multiple of 8")
    units = -(-m // align)
    base, extra = divmod(units, world)
    blocks, row = [], 0
    for r in range(world):
        n_units = base + (1 if r < extra else 0)
        rows = min(n_units * align, m - row)
        blocks.append(RowBlock(r, world, row, max(rows, 0), m))
        row += max(rows, 0)
    if row != m:
        raise AssertionError("row blocks do not cover M")
    return blocks


def max_rows(blocks: list[RowBlock]) -> int:
    return max(b.rows for b in blocks)


def relayout(gathered, blocks: list[RowBlock], n: int, out=None):
    """Place gathered per-rank column-major blocks into the global C.

    gathered: tensor viewable as [P][n][pad_rows] (each rank's C block with
    leading dimension pad_rows = max block rows); returns/fills out, a tensor
    of shape (n, M) whose row-major storage is the column-major C."""
    import torch

    world = len(blocks)
    pad = max_rows(blocks)
    m = blocks[0].m
    g = gathered.reshape(world, n, pad)
    if out is None:
        out = torch.empty((n, m), dtype=gathered.dtype, device=gathered.device)
    for b in blocks:
        if b.rows:
            out[:, b.row0:b.row0 + b.rows].copy_(g[b.rank, :, :b.rows])
    return out


def gather_c(c_local, blocks: list[RowBlock], n: int, group=None, out=None):
    """All-gather every rank's C block (shape (n, pad_rows), column-major with
    leading dimension pad_rows) and re-lay them out into the global C."""
    import torch
    import torch.distributed as dist

    pad = max_rows(blocks)
    if tuple(c_local.shape) != (n, pad):
        raise ValueError(f"local C block must be ({n}, {pad})")
    world = len(blocks)
    flat = c_local.contiguous().reshape(-1)
    gathered = torch.empty((world * n * pad,), dtype=c_local.dtype, device=c_local.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(gathered, flat, group=group)
    else:  # gloo: list form
        parts = list(gathered.chunk(world))
        dist.all_gather(parts, flat, group=group)
        gathered = torch.cat(parts)
    return relayout(gathered, blocks, n, out)


class ShardedGemm:
    """This rank's share of a row-block-sharded GEMM on its current GPU.

    Allocates A (its rows, padded to the common block height so every rank's
    C block has the same leading dimension), B (replicated) and C, fills the
    inputs with the counter-based generator (mode 4 uniform[-1,1] by default)
    and prepares the kernel through the C ABI."""

    def __init__(self, m, n, k, layout, rank, world, mode=4, seed=0, align=DEFAULT_ALIGN,
                 variant=0, device=None):
        import torch

        import bmgemm as bm

        self.blocks = row_blocks(m, world, align)
        self.block = self.blocks[rank]
        self.m, self.n, self.k, self.layout = m, n, k, layout.upper()
        self.pad = max_rows(self.blocks)
        rows = self.block.rows
        dev = device or torch.device("cuda", torch.cuda.current_device())
        pad = self.pad
        if self.layout == "NT":
            a = torch.zeros((k, pad), dtype=torch.float16, device=dev)
            b = torch.empty((k, n), dtype=torch.float16, device=dev)
            if rows:
                bm.fill(a, rows, k, row_major=False, mode=mode, seed=seed, matrix_id=0,
                        row0=self.block.row0, full_ld=m, ld=pad)
            bm.fill(b, n, k, row_major=False, mode=mode, seed=seed, matrix_id=1)
            lda, ldb = pad, n
        elif self.layout == "TN":
            a = torch.zeros((pad, k), dtype=torch.float16, device=dev)
            b = torch.empty((n, k), dtype=torch.float16, device=dev)
            if rows:
                bm.fill(a, rows, k, row_major=True, mode=mode, seed=seed, matrix_id=0,
                        row0=self.block.row0, full_ld=k)
            bm.fill(b, n, k, row_major=True, mode=mode, seed=seed, matrix_id=1)
            lda, ldb = k, k
        else:
            raise ValueError("layout must be NT or TN")
        self.a, self.b = a, b
        self.c = torch.zeros((n, pad), dtype=torch.float16, device=dev)
        self.gemm = None
        if rows:
            self.gemm = bm.Gemm(rows, n, k, self.layout, a.data_ptr(), b.data_ptr(),
                                self.c.data_ptr(), lda=lda, ldb=ldb, ldc=pad, variant=variant)

    @property
    def flops(self) -> float:
        return 2.0 * self.block.rows * self.n * self.k

    def launch(self, stream=None) -> None:
        if self.gemm is not None:
            self.gemm.launch(stream)

    def gather(self, group=None, out=None):
        return gather_c(self.c, self.blocks, self.n, group=group, out=out)

    def close(self) -> None:
        if self.gemm is not None:
            self.gemm.close()
            self.gemm = None
