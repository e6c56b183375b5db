"""kairo_b200.ops: the block-sparse SpMM operators (CUDA only).

Mirrors the reference's ``kairo.ops`` export surface (kairo/ops/
__init__.py:5-17): ``block_sparse_mm``, ``sparse_gather``,
``sparse_scatter_grad`` and ``cuda_ext_available``, plus the BSR-level
operators of this package.
"""

from __future__ import annotations

from kairo_b200.ops._autotuner import TileAutotuner, TileConfig
from kairo_b200.ops.embedding import MaskRows, sort_mask_rows, sparse_gather, sparse_scatter_grad
from kairo_b200.ops.backward import (
    BlockSparseLinear,
    TransposedBsr,
    bsr_transpose,
    sparse_linear_backward,
    sparse_linear_weight_grad,
    transpose_values,
)
from kairo_b200.ops.spmm import (
    KernelConfig,
    RowGroups,
    block_sparse_mm,
    block_sparse_mm_bsr,
    bsr_from_mask,
    bsr_from_tiles,
    bsr_row_groups,
    describe,
    pending_device_error,
    sparse_linear,
)


def cuda_ext_available() -> bool:
    """True if the native library (libkairo_spmm.so) is built and loadable.

    Same role as the reference's check of ``kairo._C``
    (kairo/ops/sparse_embedding.py:14-20)."""
    from kairo_b200 import _lib

    return _lib.available()


__all__ = [
    "cuda_ext_available",
    "block_sparse_mm",
    "block_sparse_mm_bsr",
    "bsr_from_mask",
    "bsr_from_tiles",
    "bsr_row_groups",
    "RowGroups",
    "describe",
    "pending_device_error",
    "sparse_linear",
    "KernelConfig",
    "BlockSparseLinear",
    "TransposedBsr",
    "bsr_transpose",
    "sparse_linear_backward",
    "sparse_linear_weight_grad",
    "transpose_values",
    "TileAutotuner",
    "TileConfig",
    "MaskRows",
    "sort_mask_rows",
    "sparse_gather",
    "sparse_scatter_grad",
]
