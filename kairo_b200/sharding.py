"""Multi-GPU BSR SpMM: nnz-balanced block-row sharding, B replicated.

One process per GPU.  The sparse A is cut into contiguous block-row ranges of
about equal nonzero-block count (``partition_rows``, the C-ABI
``kairo_partition_rows``); every rank holds the full B and computes its own
rows of C with the single-GPU kernel, so the compute path has no collective.
Only when the caller wants the whole C on every rank is an all-gather run
(``gather_rows``: NCCL over NVLink for CUDA tensors, gloo for CPU tensors).

Optionally (``ShardedSpmm(a, n=N)``) the ranks form a (row groups x column
slices) grid instead, chosen by ``grid_shape``: each rank takes the block-rows of its row group and the columns of
its slice of B and C.  Every rank must still read, once per sweep of its
columns, the B panels its blocks touch, which on a uniform mask is all of
them; a column slice cuts that compulsory B traffic by the number of slices
(537 MB -> 268 MB per rank for the 262144^2 case at 8 GPUs, 4 x 2 grid) at
the price of a larger share of A per rank; ``grid_shape`` balances the two.
The work stays independent per rank.

The reference has no multi-GPU code; this module is the sharding layer of the
SpMM path (shard, compute, optional gather).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist

from kairo_b200 import _lib
from kairo_b200.types import BlockSparseMatrix


@dataclass(frozen=True)
class RowShard:
    """Block-rows [row_begin, row_end) of a sharded matrix, and their blocks
    [nnz_begin, nnz_end) in BSR order."""

    rank: int
    world_size: int
    row_begin: int
    row_end: int
    nnz_begin: int
    nnz_end: int
    block_rows: int  # bm

    @property
    def rows(self) -> tuple[int, int]:
        """Element rows [begin, end) of C owned by this shard (unclipped)."""
        return self.row_begin * self.block_rows, self.row_end * self.block_rows


def partition_rows(row_ptr: torch.Tensor, parts: int) -> list[int]:
    """Contiguous block-row bounds (parts + 1 entries) with about nnzb/parts
    blocks each: bounds[p] = lower_bound(row_ptr, p * nnzb / parts)."""
    if parts <= 0:
        raise ValueError("parts must be positive")
    rp = row_ptr.detach().to("cpu", torch.int64).contiguous()
    nbr = rp.numel() - 1
    bounds = (ctypes.c_int32 * (parts + 1))()
    _lib.check(_lib.lib().kairo_partition_rows(ctypes.cast(rp.data_ptr(), ctypes.POINTER(ctypes.c_int64)), nbr,
                                               parts, bounds), "kairo_partition_rows")
    return [int(b) for b in bounds]


def shard_bsr(a: BlockSparseMatrix, rank: int, world_size: int,
              bounds: list[int] | None = None) -> tuple[BlockSparseMatrix, RowShard]:
    """This rank's rows of ``a`` as a BlockSparseMatrix (row_ptr rebased,
    blocks sliced when they are stored in BSR order, else indexed through
    blk_idx), plus its RowShard."""
    if bounds is None:
        bounds = partition_rows(a.row_ptr, world_size)
    r0, r1 = bounds[rank], bounds[rank + 1]
    rp = a.row_ptr
    n0 = int(rp[r0].item())
    n1 = int(rp[r1].item())
    bm, bk = a.block_size
    m, k = a.shape
    rows = max(0, min(m, r1 * bm) - r0 * bm)
    sub_rp = (rp[r0:r1 + 1] - n0).to(torch.int32).contiguous()
    col = a.col_idx[n0:n1]
    if a.blk_idx is None:
        blocks = a.blocks[n0:n1]
        blk = None
    else:
        blocks = a.blocks
        blk = a.blk_idx[n0:n1]
    shard = BlockSparseMatrix(row_ptr=sub_rp, col_idx=col, blocks=blocks, shape=(rows, k), block_size=(bm, bk),
                              blk_idx=blk, max_row_blocks=a.max_row_blocks)
    return shard, RowShard(rank, world_size, r0, r1, n0, n1, bm)


def grid_shape(world_size: int, n: int, min_cols: int = 256, a_bytes: int | None = None,
               b_bytes: int | None = None) -> tuple[int, int]:
    """(row groups, column slices) for ``world_size`` ranks and N columns of
    C.  Column slices are powers of two dividing world_size that leave every
    rank at least ``min_cols`` columns.  Given the sizes of A (blocks and
    indices) and B, the shape minimises the bytes one rank holds and reads
    at least once, A / row_groups + B / column_slices (what its compulsory
    DRAM reads and its host uploads scale with); without them it takes the
    most column slices.  For the 262144^2 case (A 687 MB, B 537 MB, N 1024)
    that is 2 x 1, 2 x 2 and 4 x 2 at 2, 4 and 8 ranks."""
    if world_size <= 0:
        raise ValueError("world_size must be positive")
    options = [1]
    while world_size % (2 * options[-1]) == 0 and n // (2 * options[-1]) >= min_cols:
        options.append(2 * options[-1])
    if a_bytes is None or b_bytes is None:
        pc = options[-1]
    else:
        # ties go to fewer column slices (the plain row split)
        pc = min(options, key=lambda c: (a_bytes * c + b_bytes * (world_size // c), c))
    return world_size // pc, pc


def column_range(n: int, parts: int, index: int, align: int = 128) -> tuple[int, int]:
    """Columns [c0, c1) of slice ``index`` of ``parts``, cut at multiples of
    ``align`` (whole kernel column tiles, 16-byte aligned B rows)."""
    if not 0 <= index < parts:
        raise ValueError("index outside [0, parts)")
    units = (n + align - 1) // align
    return min(n, (index * units // parts) * align), min(n, ((index + 1) * units // parts) * align)


def grid_coords(rank: int, world_size: int, n: int, min_cols: int = 256, a_bytes: int | None = None,
                b_bytes: int | None = None) -> tuple[int, int, int, int]:
    """(row group, column slice, row groups, column slices) of ``rank``."""
    pr, pc = grid_shape(world_size, n, min_cols, a_bytes, b_bytes)
    return rank // pc, rank % pc, pr, pc


def operand_bytes(a: BlockSparseMatrix, n: int) -> tuple[int, int]:
    """(bytes of A's blocks and indices, bytes of a (K x n) B in A's dtype)."""
    bm, bk = a.block_size
    es = a.blocks.element_size()
    return a.nnzb * (bm * bk * es + 4) + (a.nbr + 1) * 4, a.shape[1] * n * es


def gather_rows(c_local: torch.Tensor, bounds: list[int], block_rows: int, total_rows: int,
                group=None) -> torch.Tensor:
    """All-gather row shards of C (unequal sizes) into the full (total_rows, N)
    matrix on every rank.  Shards are padded to the largest one for a single
    all_gather_into_tensor, then trimmed."""
    world = dist.get_world_size(group)
    n = c_local.shape[1]
    sizes = [max(0, min(total_rows, bounds[p + 1] * block_rows) - bounds[p] * block_rows) for p in range(world)]
    pad = max(sizes) if sizes else 0
    buf = torch.zeros(pad, n, dtype=c_local.dtype, device=c_local.device)
    buf[: c_local.shape[0]] = c_local
    if c_local.is_cuda:
        out = torch.empty(world * pad, n, dtype=c_local.dtype, device=c_local.device)
        dist.all_gather_into_tensor(out, buf, group=group)
        parts = [out[p * pad: p * pad + sizes[p]] for p in range(world)]
    else:
        bufs = [torch.empty_like(buf) for _ in range(world)]
        dist.all_gather(bufs, buf, group=group)
        parts = [bufs[p][: sizes[p]] for p in range(world)]
    return torch.cat(parts, dim=0)


def gather_grid(c_local: torch.Tensor, bounds: list[int], block_rows: int, total_rows: int, n: int,
                row_groups: int, col_slices: int, group=None) -> torch.Tensor:
    """All-gather the (row group x column slice) tiles of C into the full
    (total_rows, n) matrix on every rank (rank = row group * col_slices +
    slice).  Tiles are padded to the largest one for one all-gather."""
    world = dist.get_world_size(group)
    rows = [max(0, min(total_rows, bounds[g + 1] * block_rows) - bounds[g] * block_rows) for g in range(row_groups)]
    cols = [column_range(n, col_slices, j) for j in range(col_slices)]
    pr_max = max(rows) if rows else 0
    pc_max = max(c1 - c0 for c0, c1 in cols) if cols else 0
    buf = torch.zeros(pr_max, pc_max, dtype=c_local.dtype, device=c_local.device)
    buf[: c_local.shape[0], : c_local.shape[1]] = c_local
    if c_local.is_cuda:
        out = torch.empty(world * pr_max, pc_max, dtype=c_local.dtype, device=c_local.device)
        dist.all_gather_into_tensor(out, buf, group=group)
        tiles = [out[r * pr_max:(r + 1) * pr_max] for r in range(world)]
    else:
        tiles = [torch.empty_like(buf) for _ in range(world)]
        dist.all_gather(tiles, buf, group=group)
    full = torch.empty(total_rows, n, dtype=c_local.dtype, device=c_local.device)
    for r in range(world):
        g, j = divmod(r, col_slices)
        r0 = bounds[g] * block_rows
        c0, c1 = cols[j]
        full[r0:r0 + rows[g], c0:c1] = tiles[r][: rows[g], : c1 - c0]
    return full


class ShardedSpmm:
    """C = A @ B with A sharded by block-rows over the ranks of ``group``.

    ``compute`` runs one rank's SpMM (default: the CUDA kernel through
    ``block_sparse_mm_bsr``); ``forward(B)`` returns this rank's rows of C, or
    the full C on every rank with ``gather=True``.  With ``n`` given (the
    columns of B and C) the ranks form the ``grid_shape`` grid: each takes its
    row group's block-rows and its column slice, ``forward`` returns that
    tile of C, and ``gather=True`` assembles the whole C.
    """

    def __init__(self, a: BlockSparseMatrix, group=None,
                 compute: Callable[[BlockSparseMatrix, torch.Tensor], torch.Tensor] | None = None,
                 n: int | None = None) -> None:
        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.n = n
        if n is None:
            self.row_groups, self.col_slices, self.row_group, self.col_slice = self.world, 1, self.rank, 0
        else:
            self.row_group, self.col_slice, self.row_groups, self.col_slices = grid_coords(
                self.rank, self.world, n, 256, *operand_bytes(a, n))
        self.bounds = partition_rows(a.row_ptr, self.row_groups)
        self.local, self.shard = shard_bsr(a, self.row_group, self.row_groups, self.bounds)
        self.columns = column_range(n, self.col_slices, self.col_slice) if n is not None else None
        self.total_rows = a.shape[0]
        if compute is None:
            from kairo_b200.ops.spmm import block_sparse_mm_bsr

            compute = block_sparse_mm_bsr
        self._compute = compute

    def forward(self, B: torch.Tensor, gather: bool = False) -> torch.Tensor:
        if self.columns is not None:
            if B.shape[1] != self.n:
                raise ValueError(f"B must have {self.n} columns")
            c0, c1 = self.columns
            c_local = self._compute(self.local, B[:, c0:c1])
            if not gather or self.world == 1:
                return c_local
            return gather_grid(c_local, self.bounds, self.shard.block_rows, self.total_rows, self.n,
                               self.row_groups, self.col_slices, self.group)
        c_local = self._compute(self.local, B)
        if not gather or self.world == 1:
            return c_local
        return gather_rows(c_local, self.bounds, self.shard.block_rows, self.total_rows, self.group)
