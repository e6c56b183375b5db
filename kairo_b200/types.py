"""Frozen domain types of the block-sparse SpMM path.

``SparseMask`` keeps the reference's field names and behaviour
(kairo/types.py:10-40): a COO list of active positions, here used at tile
granularity as the ``block_mask`` argument of ``block_sparse_mm``.

``BlockSparseMatrix`` is the BSR form the kernels consume (the reference has
no row-pointer type; its only row-offset construction is
kairo/ops/sparse_embedding.py:23-56, whose stable-sort convention the
device builder reproduces).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class SparseMask:
    """Immutable sparse mask in COO format.

    Attributes:
        indices: (2, nnz) int64 tensor of [row; column] positions (tile
            positions when used as a block mask).
        values: (nnz,) tensor of values at the active positions (ones).
        dense_shape: shape of the dense grid (rows, cols).
        sparsity_ratio: fraction of inactive positions (0.0 dense, 1.0 empty).
    """

    indices: torch.Tensor
    values: torch.Tensor
    dense_shape: tuple[int, int]
    sparsity_ratio: float

    def to_dense(self) -> torch.Tensor:
        """Dense tensor of the mask (values scattered at the indices)."""
        dense = torch.zeros(self.dense_shape, dtype=self.values.dtype, device=self.values.device)
        dense[self.indices[0], self.indices[1]] = self.values
        return dense

    @property
    def nnz(self) -> int:
        """Number of active positions."""
        return self.indices.shape[1]

    @property
    def device(self) -> torch.device:
        """Device of the mask tensors."""
        return self.indices.device


@dataclass(frozen=True)
class BlockSparseMatrix:
    """A block-sparse matrix in BSR form, resident on one CUDA device.

    Attributes:
        row_ptr: (nbr + 1,) int32, offsets of each block-row's blocks.
        col_idx: (nnzb,) int32, block-column of every block, in row order.
        blocks: (n_stored, bm, bk) dense block storage (float32/float16/bfloat16).
        shape: logical (M, K) of the matrix.
        block_size: (bm, bk).
        blk_idx: optional (nnzb,) int32; block p is ``blocks[blk_idx[p]]``.
            ``None`` means block p is ``blocks[p]``.
        max_row_blocks: length of the longest block-row, when known (0 =
            unknown).  A scheduling hint: the band schedule is chosen
            automatically only when it shows rows of similar length.
            ``bsr_from_tiles`` fills it in; ``shard_bsr`` carries it over.
    """

    row_ptr: torch.Tensor
    col_idx: torch.Tensor
    blocks: torch.Tensor
    shape: tuple[int, int]
    block_size: tuple[int, int]
    blk_idx: torch.Tensor | None = None
    max_row_blocks: int = 0

    def __post_init__(self) -> None:
        m, k = self.shape
        bm, bk = self.block_size
        if m < 0 or k < 0:
            raise ValueError(f"shape must be non-negative, got {self.shape}")
        if bm <= 0 or bk <= 0:
            raise ValueError(f"block_size must be positive, got {self.block_size}")
        nbr = (m + bm - 1) // bm
        if self.row_ptr.dim() != 1 or self.row_ptr.numel() != nbr + 1:
            raise ValueError(f"row_ptr must have {nbr + 1} entries, got {tuple(self.row_ptr.shape)}")
        if self.row_ptr.dtype != torch.int32 or self.col_idx.dtype != torch.int32:
            raise ValueError("row_ptr and col_idx must be int32")
        if self.blk_idx is not None and self.blk_idx.dtype != torch.int32:
            raise ValueError("blk_idx must be int32")
        if self.blocks.dim() != 3 or tuple(self.blocks.shape[1:]) != (bm, bk):
            raise ValueError(f"blocks must be (n, {bm}, {bk}), got {tuple(self.blocks.shape)}")
        if self.blk_idx is None and self.blocks.shape[0] < self.col_idx.numel():
            raise ValueError("fewer stored blocks than nonzero blocks")
        if self.max_row_blocks < 0:
            raise ValueError("max_row_blocks must be non-negative")

    @property
    def nbr(self) -> int:
        return self.row_ptr.numel() - 1

    @property
    def nbc(self) -> int:
        return (self.shape[1] + self.block_size[1] - 1) // self.block_size[1]

    @property
    def nnzb(self) -> int:
        return self.col_idx.numel()

    @property
    def dtype(self) -> torch.dtype:
        return self.blocks.dtype

    @property
    def device(self) -> torch.device:
        return self.blocks.device

    @property
    def sparsity(self) -> float:
        total = self.nbr * self.nbc
        return 1.0 - self.nnzb / total if total else 0.0
