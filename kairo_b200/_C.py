"""Python-visible extension functions, mirroring the reference's ``kairo._C``.

The reference builds a pybind11 module (csrc/bindings.cpp:109-125); here the
same function names are thin wrappers over the C ABI of libkairo_spmm, with
the reference's argument checks and messages (bindings.cpp:92-100,
csrc/acc_spmm_kernel.cu:166-167) raised as ``RuntimeError``.
"""

from __future__ import annotations

import ctypes

import torch

from kairo_b200 import _lib


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def acc_spmm_forward(
    A_tiles: torch.Tensor,
    tile_row_ids: torch.Tensor,
    tile_col_ids: torch.Tensor,
    B: torch.Tensor,
    M: int,
    K: int,
    N: int,
    num_tiles: int,
    tile_m: int,
    tile_k: int,
) -> torch.Tensor:
    """Block-sparse tiled matmul forward (CUDA).

    C (M x N, fp32) = sum over tiles t of A_tiles[t] placed at block
    (tile_row_ids[t], tile_col_ids[t]) times B.  Same arguments and result as
    the reference's ``kairo._C.acc_spmm_forward`` (bindings.cpp:84-103 ->
    acc_spmm_kernel.cu:158-207); tiles may be in any order.  Accepts float32,
    float16 and bfloat16 tiles (A_tiles and B of one dtype).
    """
    _require(A_tiles.is_contiguous(), "A_tiles must be contiguous")
    _require(tile_row_ids.is_contiguous(), "tile_row_ids must be contiguous")
    _require(tile_col_ids.is_contiguous(), "tile_col_ids must be contiguous")
    _require(B.is_contiguous(), "B must be contiguous")
    _require(tile_row_ids.dtype == torch.int32, "tile_row_ids must be int32")
    _require(tile_col_ids.dtype == torch.int32, "tile_col_ids must be int32")
    _require(M > 0 and K > 0 and N > 0, "dimensions must be positive")
    _require(A_tiles.is_cuda, "A_tiles must be on CUDA")
    _require(B.is_cuda, "B must be on CUDA")
    _require(A_tiles.dtype == B.dtype, "A_tiles and B must have the same dtype")
    _require(tuple(B.shape) == (K, N), f"B must be ({K}, {N}), got {tuple(B.shape)}")
    _require(tile_row_ids.numel() == num_tiles and tile_col_ids.numel() == num_tiles,
             "tile id arrays must hold num_tiles entries")
    _require(A_tiles.numel() == num_tiles * tile_m * tile_k, "A_tiles must be (num_tiles, tile_m, tile_k)")
    dt = _lib.kairo_dtype(A_tiles.dtype)
    lib = _lib.lib()
    device = B.device
    with torch.cuda.device(device):
        C = torch.empty(M, N, dtype=torch.float32, device=device)
        nbytes = ctypes.c_size_t(0)
        _lib.check(lib.kairo_acc_spmm_forward_workspace_size(M, K, N, num_tiles, tile_m, tile_k, dt,
                                                             ctypes.byref(nbytes)),
                   "acc_spmm_forward")
        ws = _lib.workspace(nbytes.value, device)
        _lib.check(lib.kairo_acc_spmm_forward(
            A_tiles.data_ptr() if num_tiles else None, tile_row_ids.data_ptr() if num_tiles else None,
            tile_col_ids.data_ptr() if num_tiles else None, B.data_ptr(), C.data_ptr(), M, K, N, num_tiles,
            tile_m, tile_k, dt, ws.data_ptr(), ws.numel(), _lib.stream_handle(device)), "acc_spmm_forward")
    return C


def sparse_gather_forward(
    weight: torch.Tensor,
    mask_rows: torch.Tensor,
    mask_cols: torch.Tensor,
    batch_ids: torch.Tensor,
    row_offsets: torch.Tensor,
) -> torch.Tensor:
    """Masked embedding gather (CUDA): out[b] = weight[batch_ids[b]] on the
    row's active columns (mask_cols[row_offsets[r]:row_offsets[r+1]]), zero
    elsewhere and for ids outside [0, N).  Same arguments, checks and result
    as the reference's ``kairo._C.sparse_gather_forward`` (bindings.cpp:39-61
    -> sparse_embedding_kernel.cu:135-184); weight may also be float16 or
    bfloat16."""
    _require(weight.is_contiguous(), "weight must be contiguous")
    _require(mask_rows.is_contiguous(), "mask_rows must be contiguous")
    _require(mask_cols.is_contiguous(), "mask_cols must be contiguous")
    _require(batch_ids.is_contiguous(), "batch_ids must be contiguous")
    _require(row_offsets.is_contiguous(), "row_offsets must be contiguous")
    _require(weight.dtype in (torch.float32, torch.float16, torch.bfloat16),
             "weight must be float32 (or float16 / bfloat16)")
    _require(mask_rows.dtype == torch.int64, "mask_rows must be int64")
    _require(mask_cols.dtype == torch.int64, "mask_cols must be int64")
    _require(batch_ids.dtype == torch.int64, "batch_ids must be int64")
    _require(weight.is_cuda, "weight must be on CUDA")
    _require(weight.dim() == 2, "weight must be 2D")
    _require(batch_ids.is_cuda, "batch_ids must be on CUDA")
    _require(row_offsets.dtype == torch.int64 and row_offsets.numel() >= weight.shape[0] + 1,
             "row_offsets must be int64 with N + 1 entries")
    n, d = weight.shape
    b = batch_ids.numel()
    nnz = mask_cols.numel()
    out = torch.empty(b, d, dtype=weight.dtype, device=weight.device)
    if b == 0:
        return out
    with torch.cuda.device(weight.device):
        _lib.check(_lib.lib().kairo_sparse_gather(weight.data_ptr(), n, d, _lib.kairo_dtype(weight.dtype),
                                                  row_offsets.data_ptr(), mask_cols.data_ptr() if nnz else None, nnz,
                                                  batch_ids.data_ptr(), b, out.data_ptr(),
                                                  _lib.stream_handle(weight.device)), "sparse_gather_forward")
    return out


def sparse_scatter_backward(
    grad_output: torch.Tensor,
    active_ids: torch.Tensor,
    batch_ids: torch.Tensor,
    N: int,
    D: int,
) -> torch.Tensor:
    """Sparse gradient scatter (CUDA): (N, D), row active_ids[s] = sum of
    grad_output[b] over batch_ids[b] == active_ids[s], zero elsewhere.  Same
    arguments, checks and result as the reference's
    ``kairo._C.sparse_scatter_backward`` (bindings.cpp:63-82 ->
    sparse_embedding_kernel.cu:186-219), summed deterministically in batch
    order; grad_output may also be float16 or bfloat16."""
    _require(grad_output.is_contiguous(), "grad_output must be contiguous")
    _require(active_ids.is_contiguous(), "active_ids must be contiguous")
    _require(batch_ids.is_contiguous(), "batch_ids must be contiguous")
    _require(grad_output.dtype in (torch.float32, torch.float16, torch.bfloat16),
             "grad_output must be float32 (or float16 / bfloat16)")
    _require(active_ids.dtype == torch.int64, "active_ids must be int64")
    _require(batch_ids.dtype == torch.int64, "batch_ids must be int64")
    _require(N > 0, "N must be positive")
    _require(D > 0, "D must be positive")
    _require(grad_output.is_cuda, "grad_output must be on CUDA")
    _require(active_ids.is_cuda, "active_ids must be on CUDA")
    _require(batch_ids.is_cuda, "batch_ids must be on CUDA")
    _require(grad_output.numel() == batch_ids.numel() * D, "grad_output must be (B, D)")
    from kairo_b200.ops.embedding import sparse_scatter_grad

    return sparse_scatter_grad(grad_output.view(batch_ids.numel(), D), active_ids, batch_ids, N, D)
