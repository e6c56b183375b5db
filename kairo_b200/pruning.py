"""Block-granular magnitude pruning and gradient-based regrowth on the device.

Mirrors the reference's mask topology updates (kairo/training/sparse_rec/
topology.py), which work element by element, at block granularity for a
BSR weight:

* ``prune_blocks`` -- ``prune_mask`` (topology.py:50-118): keep the
  ``nnzb - int(nnzb * fraction)`` blocks of largest L2 norm, in their BSR
  order.
* ``grow_blocks`` -- ``grow_mask`` (topology.py:121-189): activate the
  inactive blocks with the largest scores (e.g. accumulated gradient norms),
  new blocks zero; active blocks score -1 as in the reference.
* ``update_blocks`` -- ``update_topology`` (topology.py:192-232): prune, then
  grow back as many as were pruned.
* ``block_magnitude_mask`` -- a SparseMask of the top fraction of a dense
  weight's blocks by L2 norm, indices sorted (how the linear-layer
  workload's mask is defined).

Scores come from ``kairo_block_norms`` / ``kairo_bsr_block_norms`` and the
selection from ``kairo_topk_indices`` (a radix select); bookkeeping of the
block lists is plain tensor indexing.  One difference from the reference:
grown blocks are appended in ascending block index order, where
``grow_mask`` appends them in descending score order; the selected set is
the same.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
from torch import Tensor

from kairo_b200 import _lib
from kairo_b200.ops.spmm import _bsr_desc, _require_cuda
from kairo_b200.types import BlockSparseMatrix, SparseMask


def _pair(block) -> tuple[int, int]:
    return (int(block), int(block)) if isinstance(block, int) else (int(block[0]), int(block[1]))


def block_norms(A: Tensor, block) -> Tensor:
    """L2 norm of every block of a dense CUDA matrix: (nbr, nbc) fp32."""
    _require_cuda(A, op="block_norms")
    if A.dim() != 2:
        raise ValueError("A must be 2-D")
    if A.stride(1) != 1:
        A = A.contiguous()
    bm, bk = _pair(block)
    m, k = A.shape
    nbr, nbc = (m + bm - 1) // bm, (k + bk - 1) // bk
    out = torch.empty(nbr, nbc, dtype=torch.float32, device=A.device)
    with torch.cuda.device(A.device):
        _lib.check(_lib.lib().kairo_block_norms(A.data_ptr(), m, k, A.stride(0), bm, bk, _lib.kairo_dtype(A.dtype),
                                                out.data_ptr(), _lib.stream_handle(A.device)), "block_norms")
    return out


def bsr_block_norms(W: BlockSparseMatrix) -> Tensor:
    """L2 norm of every block of W, in BSR order: (nnzb,) fp32."""
    _require_cuda(W.blocks, op="bsr_block_norms")
    out = torch.empty(W.nnzb, dtype=torch.float32, device=W.device)
    if W.nnzb:
        desc = _bsr_desc(W)
        with torch.cuda.device(W.device):
            _lib.check(_lib.lib().kairo_bsr_block_norms(ctypes.byref(desc), out.data_ptr(),
                                                        _lib.stream_handle(W.device)), "bsr_block_norms")
    return out


def topk_indices(scores: Tensor, count: int) -> Tensor:
    """Indices of the ``count`` largest scores, ascending (int64); ties at the
    threshold go to the lower index, NaN ranks lowest."""
    _require_cuda(scores, op="topk_indices")
    s = scores.reshape(-1).to(torch.float32).contiguous()
    n = s.numel()
    if count < 0 or count > n:
        raise ValueError(f"count must be in [0, {n}], got {count}")
    out = torch.empty(count, dtype=torch.int64, device=s.device)
    if count == 0:
        return out
    lib = _lib.lib()
    with torch.cuda.device(s.device):
        nbytes = ctypes.c_size_t(0)
        _lib.check(lib.kairo_topk_workspace_size(n, ctypes.byref(nbytes)), "topk_indices")
        ws = torch.empty(max(nbytes.value, 256), dtype=torch.uint8, device=s.device)
        _lib.check(lib.kairo_topk_indices(s.data_ptr(), n, count, out.data_ptr(), ws.data_ptr(), ws.numel(),
                                          _lib.stream_handle(s.device)), "topk_indices")
    return out


def block_magnitude_mask(W: Tensor, block: int, keep_fraction: float) -> SparseMask:
    """SparseMask (block grid) of the ``int(nblocks * keep_fraction)`` blocks
    of a dense weight with the largest L2 norms, indices in row-major order."""
    norms = block_norms(W, block)
    nbr, nbc = norms.shape
    total = nbr * nbc
    keep = int(total * keep_fraction)
    idx = topk_indices(norms, keep)
    indices = torch.stack([idx // nbc, idx % nbc], dim=0)
    return SparseMask(indices=indices, values=torch.ones(keep, device=W.device), dense_shape=(nbr, nbc),
                      sparsity_ratio=1.0 - keep / total if total else 0.0)


def _rows_of(W: BlockSparseMatrix) -> Tensor:
    counts = (W.row_ptr[1:] - W.row_ptr[:-1]).to(torch.int64)
    return torch.repeat_interleave(torch.arange(W.nbr, device=W.device), counts)


def _from_positions(W: BlockSparseMatrix, rows: Tensor, cols: Tensor, blocks: Tensor) -> BlockSparseMatrix:
    """BSR matrix from block lists already in BSR order (rows non-decreasing)."""
    counts = torch.bincount(rows, minlength=W.nbr) if rows.numel() else torch.zeros(W.nbr, dtype=torch.int64,
                                                                                       device=W.device)
    row_ptr = torch.zeros(W.nbr + 1, dtype=torch.int32, device=W.device)
    row_ptr[1:] = torch.cumsum(counts, 0).to(torch.int32)
    longest = int(counts.max()) if counts.numel() else 0
    return BlockSparseMatrix(row_ptr=row_ptr, col_idx=cols.to(torch.int32).contiguous(), blocks=blocks.contiguous(),
                             shape=W.shape, block_size=W.block_size, max_row_blocks=longest)


def _stored(W: BlockSparseMatrix) -> Tensor:
    return W.blocks if W.blk_idx is None else W.blocks[W.blk_idx.long()]


def prune_blocks(W: BlockSparseMatrix, prune_fraction: float) -> BlockSparseMatrix:
    """Drop the ``int(nnzb * prune_fraction)`` blocks of smallest L2 norm."""
    if prune_fraction <= 0.0 or W.nnzb == 0 or int(W.nnzb * prune_fraction) == 0:
        return _from_positions(W, _rows_of(W), W.col_idx.clone(), _stored(W).clone())
    keep = W.nnzb - int(W.nnzb * prune_fraction)
    pos = topk_indices(bsr_block_norms(W), keep)
    return _from_positions(W, _rows_of(W)[pos], W.col_idx[pos], _stored(W)[pos])


def grow_blocks(W: BlockSparseMatrix, scores: Tensor, grow_count: int) -> BlockSparseMatrix:
    """Activate the ``grow_count`` inactive blocks with the largest ``scores``
    ((nbr, nbc), e.g. accumulated gradient norms); new blocks are zero."""
    if grow_count <= 0:
        return _from_positions(W, _rows_of(W), W.col_idx.clone(), _stored(W).clone())
    nbr, nbc = W.nbr, W.nbc
    if tuple(scores.shape) != (nbr, nbc):
        raise ValueError(f"scores must be ({nbr}, {nbc})")
    rows = _rows_of(W)
    flat = scores.to(torch.float32).reshape(-1).clone()
    active = rows * nbc + W.col_idx.long()
    flat[active] = -1.0
    inactive = nbr * nbc - W.nnzb
    grow = min(grow_count, inactive)
    if grow == 0:
        return _from_positions(W, rows, W.col_idx.clone(), _stored(W).clone())
    new = topk_indices(flat, grow)
    all_rows = torch.cat([rows, new // nbc])
    all_cols = torch.cat([W.col_idx.long(), new % nbc])
    bm, bk = W.block_size
    all_blocks = torch.cat([_stored(W), torch.zeros(grow, bm, bk, dtype=W.dtype, device=W.device)])
    order = torch.sort(all_rows, stable=True).indices  # BSR order: stable by block-row
    return _from_positions(W, all_rows[order], all_cols[order], all_blocks[order])


@dataclass(frozen=True)
class BlockUpdateResult:
    """Result of ``update_blocks`` (the block analogue of MaskUpdateResult)."""

    matrix: BlockSparseMatrix
    num_pruned: int
    num_grown: int
    score_norm: float


def update_blocks(W: BlockSparseMatrix, scores: Tensor, prune_fraction: float) -> BlockUpdateResult:
    """Prune ``prune_fraction`` of the blocks by norm, then grow back as many
    from the highest-scoring inactive blocks."""
    pruned = prune_blocks(W, prune_fraction)
    n_pruned = W.nnzb - pruned.nnzb
    grown = grow_blocks(pruned, scores, n_pruned)
    return BlockUpdateResult(matrix=grown, num_pruned=n_pruned, num_grown=grown.nnzb - pruned.nnzb,
                             score_norm=float(scores.float().norm().item()))
