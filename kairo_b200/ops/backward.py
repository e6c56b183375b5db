"""Backward pass of the block-sparse linear layer ``Y = X @ W^T``.

The reference has no backward for its SpMM; this module adds the one a
sparse-training caller of ``sparse_linear`` needs, with W's sparsity fixed:

* ``dX = dY @ W`` -- the same LINEAR-layout SpMM on the transposed weight,
  ``sparse_linear(dY, W^T)``; W^T comes from ``bsr_transpose`` (device-side,
  stable (column, row) order, blocks transposed).
* ``dW`` on W's nonzero blocks only -- ``dW[p] = dY[:, rows of p]^T @ X[:,
  cols of p]``, a block-sampled dense x dense product (``kairo_bsr_sddmm``:
  tcgen05 kernel for 64 x 64 f16/bf16 blocks, CUDA cores otherwise).

``BlockSparseLinear`` wraps both in an autograd-aware module whose parameter
is the (nnzb, bm, bk) block tensor.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
from torch import Tensor

from kairo_b200 import _lib
from kairo_b200.ops.spmm import KernelConfig, _bsr_desc, _require_cuda, sparse_linear
from kairo_b200.types import BlockSparseMatrix


@dataclass(frozen=True)
class TransposedBsr:
    """W^T of a BSR matrix W.

    matrix: W^T as a BlockSparseMatrix (blocks transposed, in W^T order);
    perm: (nnzb,) int32, W's BSR position of every W^T position.
    """

    matrix: BlockSparseMatrix
    perm: Tensor


def _scratch(nbytes: int, device: torch.device) -> Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def bsr_transpose(a: BlockSparseMatrix, *, check: bool = False, row_hint: bool = True) -> TransposedBsr:
    """W^T on the device (structure and transposed blocks).

    ``row_hint`` reads W^T's longest block-row back from the device (one
    synchronisation) into ``max_row_blocks``, the hint the SpMM scheduler
    uses to pick the band schedule; with ``row_hint=False`` the call is
    asynchronous.  ``check=True`` synchronises and raises KairoDeviceError
    on an invalid index or a block-column longer than 16384 blocks."""
    _require_cuda(a.blocks, a.row_ptr, op="bsr_transpose")
    m, k = a.shape
    bm, bk = a.block_size
    nbc = a.nbc
    dev = a.device
    lib = _lib.lib()
    desc = _bsr_desc(a)
    with torch.cuda.device(dev):
        nbytes = ctypes.c_size_t(0)
        _lib.check(lib.kairo_bsr_transpose_workspace_size(ctypes.byref(desc), ctypes.byref(nbytes)), "bsr_transpose")
        ws = _scratch(nbytes.value, dev)
        row_ptr_t = torch.empty(nbc + 1, dtype=torch.int32, device=dev)
        col_idx_t = torch.empty(a.nnzb, dtype=torch.int32, device=dev)
        perm_t = torch.empty(a.nnzb, dtype=torch.int32, device=dev)
        blocks_t = torch.empty(a.nnzb, bk, bm, dtype=a.dtype, device=dev)
        _lib.check(lib.kairo_bsr_transpose(ctypes.byref(desc), row_ptr_t.data_ptr(), _lib.ptr(col_idx_t) if a.nnzb else None,
                                           _lib.ptr(perm_t) if a.nnzb else None, _lib.ptr(blocks_t) if a.nnzb else None,
                                           ws.data_ptr(), ws.numel(), _lib.stream_handle(dev)), "bsr_transpose")
        if check:
            _lib.raise_on_device_error(ws)
        longest = 0
        if row_hint and a.nnzb:
            # the bucket sort leaves the longest bucket (W^T row) in the
            # workspace header's second flag word
            longest = int(ws[64:72].view(torch.int32)[1].item())
    wt = BlockSparseMatrix(row_ptr=row_ptr_t, col_idx=col_idx_t, blocks=blocks_t, shape=(k, m), block_size=(bk, bm),
                           max_row_blocks=longest)
    return TransposedBsr(matrix=wt, perm=perm_t)


def transpose_values(a: BlockSparseMatrix, t: TransposedBsr) -> TransposedBsr:
    """Refresh W^T's blocks from W's current values (structure unchanged)."""
    if a.nnzb == 0:
        return t
    lib = _lib.lib()
    desc = _bsr_desc(a)
    dev = a.device
    with torch.cuda.device(dev):
        ws = _scratch(256, dev)
        _lib.check(lib.kairo_bsr_transpose_values(ctypes.byref(desc), t.perm.data_ptr(), t.matrix.blocks.data_ptr(),
                                                  ws.data_ptr(), ws.numel(), _lib.stream_handle(dev)),
                   "transpose_values")
    return t


def sparse_linear_weight_grad(dY: Tensor, X: Tensor, W: BlockSparseMatrix, wt: TransposedBsr | None = None, *,
                              out_dtype: torch.dtype = torch.float32, check: bool = False) -> Tensor:
    """dW on W's nonzero blocks for Y = X @ W^T: (nnzb, bm, bk) in W's BSR
    order, ``dW[p] = dY[:, i*bm:(i+1)*bm]^T @ X[:, j*bk:(j+1)*bk]``."""
    _require_cuda(dY, X, W.blocks, op="sparse_linear_weight_grad")
    m, k = W.shape
    if dY.dim() != 2 or X.dim() != 2 or dY.shape[0] != X.shape[0] or dY.shape[1] != m or X.shape[1] != k:
        raise ValueError(f"dY must be (batch, {m}) and X (batch, {k}); got {tuple(dY.shape)} and {tuple(X.shape)}")
    if dY.dtype != W.dtype or X.dtype != W.dtype:
        raise TypeError("dY, X and W must share a dtype")
    if out_dtype not in (torch.float32, W.dtype):
        raise TypeError("dW dtype must be float32 or the weight dtype")
    if dY.stride(1) != 1:
        dY = dY.contiguous()
    if X.stride(1) != 1:
        X = X.contiguous()
    if wt is None:
        wt = bsr_transpose(W)
    bm, bk = W.block_size
    dev = W.device
    dw = torch.empty(W.nnzb, bm, bk, dtype=out_dtype, device=dev)
    if W.nnzb == 0:
        return dw
    lib = _lib.lib()
    desc = _bsr_desc(W)
    with torch.cuda.device(dev):
        nbytes = ctypes.c_size_t(0)
        _lib.check(lib.kairo_bsr_sddmm_workspace_size(ctypes.byref(desc), ctypes.byref(nbytes)), "sddmm")
        ws = _scratch(nbytes.value, dev)
        _lib.check(lib.kairo_bsr_sddmm(ctypes.byref(desc), wt.matrix.row_ptr.data_ptr(), wt.matrix.col_idx.data_ptr(),
                                       wt.perm.data_ptr(), dY.data_ptr(), dY.stride(0), X.data_ptr(), X.stride(0),
                                       X.shape[0], dw.data_ptr(), _lib.kairo_dtype(out_dtype), ws.data_ptr(),
                                       ws.numel(), _lib.stream_handle(dev)), "sparse_linear_weight_grad")
        if check:
            _lib.raise_on_device_error(ws)
    return dw


def sparse_linear_backward(dY: Tensor, X: Tensor, W: BlockSparseMatrix, wt: TransposedBsr | None = None, *,
                           need_dx: bool = True, need_dw: bool = True, dw_dtype: torch.dtype = torch.float32,
                           config: KernelConfig | None = None, check: bool = False):
    """(dX, dW) of Y = X @ W^T.  dX: (batch, in_features) in X's dtype; dW:
    (nnzb, bm, bk) in ``dw_dtype``, W's BSR order.  Either may be None."""
    if wt is None:
        wt = bsr_transpose(W)
    dX = sparse_linear(dY, wt.matrix, out_dtype=X.dtype, config=config, check=check) if need_dx else None
    dW = sparse_linear_weight_grad(dY, X, W, wt, out_dtype=dw_dtype, check=check) if need_dw else None
    return dX, dW


class _SparseLinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, X: Tensor, blocks: Tensor, module: "BlockSparseLinear") -> Tensor:
        W = module.weight_matrix(blocks)
        ctx.save_for_backward(X, blocks)
        ctx.module = module
        return sparse_linear(X, W)

    @staticmethod
    def backward(ctx, dY: Tensor):
        X, blocks = ctx.saved_tensors
        module: BlockSparseLinear = ctx.module
        W = module.weight_matrix(blocks)
        wt = transpose_values(W, module.transposed())
        dY = dY.contiguous()
        dX, dW = sparse_linear_backward(dY, X, W, wt, need_dx=ctx.needs_input_grad[0],
                                        need_dw=ctx.needs_input_grad[1], dw_dtype=blocks.dtype)
        return dX, dW, None


class BlockSparseLinear(torch.nn.Module):
    """``Y = X @ W^T`` with a block-sparse weight of fixed sparsity pattern.

    The trainable parameter is ``blocks`` (nnzb, bm, bk) in BSR order;
    ``row_ptr`` / ``col_idx`` are buffers.  Forward and both gradients run on
    this package's kernels (``sparse_linear``, ``bsr_transpose``,
    ``kairo_bsr_sddmm``)."""

    def __init__(self, W: BlockSparseMatrix) -> None:
        super().__init__()
        blocks = W.blocks if W.blk_idx is None else W.blocks[W.blk_idx.long()]
        self.blocks = torch.nn.Parameter(blocks.detach().clone())
        self.register_buffer("row_ptr", W.row_ptr.detach().clone())
        self.register_buffer("col_idx", W.col_idx.detach().clone())
        self.shape = W.shape
        self.block_size = W.block_size
        self.max_row_blocks = W.max_row_blocks
        self._wt: TransposedBsr | None = None

    def weight_matrix(self, blocks: Tensor | None = None) -> BlockSparseMatrix:
        b = self.blocks if blocks is None else blocks
        return BlockSparseMatrix(row_ptr=self.row_ptr, col_idx=self.col_idx, blocks=b.detach(), shape=self.shape,
                                 block_size=self.block_size, max_row_blocks=self.max_row_blocks)

    def transposed(self) -> TransposedBsr:
        """Cached W^T structure (its blocks are refreshed on every backward)."""
        if self._wt is None:
            self._wt = bsr_transpose(self.weight_matrix())
        return self._wt

    def forward(self, X: Tensor) -> Tensor:
        return _SparseLinearFn.apply(X, self.blocks, self)
