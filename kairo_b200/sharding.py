"""Multi-GPU BSR SpMM: nnz-balanced block-row sharding, B replicated.

One process per GPU.  The sparse A is cut into contiguous block-row ranges of
about equal nonzero-block count (``partition_rows``, the C-ABI
``kairo_partition_rows``); every rank holds the full B and computes its own
rows of C with the single-GPU kernel, so the compute path has no collective.
Only when the caller wants the whole C on every rank is an all-gather run
(``gather_rows``: NCCL over NVLink for CUDA tensors, gloo for CPU tensors).

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


class ShardedSpmm:
    """C = A @ B with A sharded by block-rows over the ranks of ``group``.

    ``compute`` runs one rank's SpMM (default: the CUDA kernel through
    ``block_sparse_mm_bsr``); ``forward(B)`` returns this rank's rows of C, or
    the full C on every rank with ``gather=True``.
    """

    def __init__(self, a: BlockSparseMatrix, group=None,
                 compute: Callable[[BlockSparseMatrix, torch.Tensor], torch.Tensor] | None = None) -> None:
        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.bounds = partition_rows(a.row_ptr, self.world)
        self.local, self.shard = shard_bsr(a, self.rank, self.world, self.bounds)
        self.total_rows = a.shape[0]
        if compute is None:
            from kairo_b200.ops.spmm import block_sparse_mm_bsr

            compute = block_sparse_mm_bsr
        self._compute = compute

    def forward(self, B: torch.Tensor, gather: bool = False) -> torch.Tensor:
        c_local = self._compute(self.local, B)
        if not gather or self.world == 1:
            return c_local
        return gather_rows(c_local, self.bounds, self.shard.block_rows, self.total_rows, self.group)
