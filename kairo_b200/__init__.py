"""kairo_b200: B200-native (sm_100a) block-sparse SpMM behind Kairo's SpMM interface.

Subpackages mirror the reference's layout for this path: ``kairo_b200.types``
(SparseMask, BlockSparseMatrix), ``kairo_b200.ops`` (block_sparse_mm,
TileAutotuner, ...), ``kairo_b200._C`` (acc_spmm_forward).  The compute runs
in libkairo_spmm.so (C ABI: include/kairo_spmm.h).
"""

__version__ = "0.1.0"

__all__ = ["__version__"]
