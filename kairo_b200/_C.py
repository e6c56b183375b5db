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
