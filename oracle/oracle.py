"""ctypes front-end of the C oracle (oracle/bsr_oracle.c).  TEST INFRASTRUCTURE.

Restates the reference's CPU path for the SpMM hot path:
  spmm_tiles      kairo/ops/spmm.py:108-134   (_block_sparse_mm_fallback)
  spmm_bsr_rows   the same arithmetic for selected block-rows of a BSR matrix
  dense_to_tiles  kairo/ops/spmm.py:16-55     (_dense_to_block_sparse)
  sort_coo_by_row kairo/ops/sparse_embedding.py:49-56
  row_offsets     kairo/ops/sparse_embedding.py:23-46
  sparse_gather   kairo/ops/sparse_embedding.py:59-101 (the CUDA kernels' values)
  sparse_scatter_grad kairo/ops/sparse_embedding.py:104-161
Pinned against fixtures generated from the reference itself (tests/golden).
Inputs are CPU torch tensors; fp16/bf16 values are widened to fp32 exactly.
"""

from __future__ import annotations

import ctypes
import subprocess
import threading
from ctypes import POINTER, c_int, c_int32, c_int64, c_void_p
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
_lib = None
_lock = threading.Lock()

_DT = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


def build(force: bool = False) -> Path:
    src = HERE / "bsr_oracle.c"
    if force or not LIB.exists() or LIB.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-B" if force else "-s", "-C", str(HERE), "liboracle.so"], check=True,
                       capture_output=True)
    return LIB


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                h = ctypes.CDLL(str(build()))
                h.oracle_spmm_tiles.restype = c_int
                h.oracle_spmm_tiles.argtypes = [c_void_p, c_int, c_void_p, c_void_p, c_int64, c_void_p, c_int,
                                                c_int64, c_int64, c_int64, c_int32, c_int32, c_void_p, c_int]
                h.oracle_spmm_bsr_rows.restype = c_int
                h.oracle_spmm_bsr_rows.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int32, c_int32,
                                                   c_void_p, c_int, c_int64, c_int64, c_int64, c_int64, c_void_p,
                                                   c_int64, c_void_p, c_int]
                h.oracle_dense_to_tiles.restype = None
                h.oracle_dense_to_tiles.argtypes = [c_void_p, c_int64, c_int64, c_int, c_void_p, c_void_p, c_int64,
                                                    c_int32, c_void_p]
                h.oracle_sort_coo_by_row.restype = c_int
                h.oracle_sort_coo_by_row.argtypes = [c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p,
                                                     c_void_p]
                h.oracle_row_offsets.restype = None
                h.oracle_row_offsets.argtypes = [c_void_p, c_int64, c_int64, c_void_p]
                h.oracle_num_threads.restype = c_int
                h.oracle_num_threads.argtypes = []
                h.oracle_bsr_sddmm.restype = c_int
                h.oracle_bsr_sddmm.argtypes = [c_void_p, c_void_p, c_int32, c_int64, c_void_p, c_int64, c_void_p,
                                               c_int64, c_int, c_int64, c_int64, c_int64, c_int32, c_int32, c_void_p,
                                               c_int]
                h.oracle_sparse_gather.restype = None
                h.oracle_sparse_gather.argtypes = [c_void_p, c_int, c_int64, c_int64, c_void_p, c_void_p, c_void_p,
                                                   c_int64, c_void_p]
                h.oracle_sparse_scatter_grad.restype = c_int
                h.oracle_sparse_scatter_grad.argtypes = [c_void_p, c_int, c_void_p, c_int64, c_void_p, c_int64,
                                                         c_int64, c_int64, c_void_p]
                h.oracle_bsr_transpose.restype = c_int
                h.oracle_bsr_transpose.argtypes = [c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_void_p, c_void_p]
                _lib = h
    return _lib


def num_threads() -> int:
    return int(load().oracle_num_threads())


def _cpu(t: torch.Tensor, dtype: torch.dtype | None = None) -> torch.Tensor:
    t = t.detach().to("cpu")
    if dtype is not None:
        t = t.to(dtype)
    return t.contiguous()


def spmm_tiles(tiles: torch.Tensor, row_ids: torch.Tensor, col_ids: torch.Tensor, B: torch.Tensor, M: int, K: int,
               N: int, tile_m: int, tile_k: int | None = None, nthreads: int = 0) -> torch.Tensor:
    """C (M x N, fp32) per _block_sparse_mm_fallback on fp32-widened inputs."""
    tile_k = tile_m if tile_k is None else tile_k
    tiles = _cpu(tiles)
    B = _cpu(B)
    r = _cpu(row_ids, torch.int32)
    c = _cpu(col_ids, torch.int32)
    if B.dim() != 2 or B.shape[0] < K or B.shape[1] < N:
        raise ValueError(f"B must be at least ({K}, {N}), got {tuple(B.shape)}")
    C = torch.empty(M, N, dtype=torch.float32)
    rc = load().oracle_spmm_tiles(tiles.data_ptr(), _DT[tiles.dtype], r.data_ptr(), c.data_ptr(), r.numel(),
                                  B.data_ptr(), _DT[B.dtype], M, K, N, tile_m, tile_k, C.data_ptr(), nthreads)
    if rc:
        raise ValueError(f"oracle_spmm_tiles failed ({rc})")
    return C


def spmm_bsr_rows(row_ptr: torch.Tensor, col_idx: torch.Tensor, blk_idx: torch.Tensor | None, blocks: torch.Tensor,
                  B: torch.Tensor, M: int, K: int, N: int, rows_sel, nthreads: int = 0) -> torch.Tensor:
    """Rows of C for the selected block-rows: ((len(rows_sel) * bm) x N) fp32."""
    rp = _cpu(row_ptr, torch.int32)
    ci = _cpu(col_idx, torch.int32)
    bi = None if blk_idx is None else _cpu(blk_idx, torch.int32)
    blocks = _cpu(blocks)
    B = _cpu(B)
    bm, bk = int(blocks.shape[1]), int(blocks.shape[2])
    if B.dim() != 2 or B.shape[0] < K or B.shape[1] < N:
        raise ValueError(f"B must be at least ({K}, {N}), got {tuple(B.shape)}")
    sel = torch.as_tensor(rows_sel, dtype=torch.int32).contiguous()
    if sel.numel() and (int(sel.min()) < 0 or int(sel.max()) >= rp.numel() - 1):
        raise ValueError("selected block-row out of range")
    out = torch.empty(sel.numel() * bm, N, dtype=torch.float32)
    rc = load().oracle_spmm_bsr_rows(rp.data_ptr(), ci.data_ptr(), None if bi is None else bi.data_ptr(),
                                     blocks.data_ptr(), _DT[blocks.dtype], bm, bk, B.data_ptr(), _DT[B.dtype],
                                     B.stride(0), M, K, N, sel.data_ptr(), sel.numel(), out.data_ptr(), nthreads)
    if rc:
        raise ValueError(f"oracle_spmm_bsr_rows failed ({rc})")
    return out


def dense_to_tiles(A: torch.Tensor, rows: torch.Tensor, cols: torch.Tensor, tile: int) -> torch.Tensor:
    A = _cpu(A)
    r = _cpu(rows, torch.int64)
    c = _cpu(cols, torch.int64)
    out = torch.empty(r.numel(), tile, tile, dtype=A.dtype)
    load().oracle_dense_to_tiles(A.data_ptr(), A.shape[0], A.shape[1], A.element_size(), r.data_ptr(), c.data_ptr(),
                                 r.numel(), tile, out.data_ptr())
    return out


def sort_coo_by_row(rows: torch.Tensor, cols: torch.Tensor, nrows: int):
    """(perm, rows_sorted, cols_sorted) as int64, stable by row."""
    r = _cpu(rows, torch.int64)
    c = _cpu(cols, torch.int64)
    perm = torch.empty_like(r)
    ro = torch.empty_like(r)
    co = torch.empty_like(c)
    rc = load().oracle_sort_coo_by_row(r.data_ptr(), c.data_ptr(), r.numel(), nrows, perm.data_ptr(), ro.data_ptr(),
                                       co.data_ptr())
    if rc:
        raise ValueError(f"oracle_sort_coo_by_row failed ({rc})")
    return perm, ro, co


def row_offsets(rows: torch.Tensor, nrows: int) -> torch.Tensor:
    r = _cpu(rows, torch.int64)
    out = torch.empty(nrows + 1, dtype=torch.int64)
    load().oracle_row_offsets(r.data_ptr(), r.numel(), nrows, out.data_ptr())
    return out


def bsr_sddmm(row_ptr: torch.Tensor, col_idx: torch.Tensor, dY: torch.Tensor, X: torch.Tensor, bm: int, bk: int,
              nthreads: int = 0) -> torch.Tensor:
    """dW blocks (nnzb, bm, bk) fp32 of Y = X @ W.T on W's nonzero blocks."""
    rp = _cpu(row_ptr, torch.int32)
    ci = _cpu(col_idx, torch.int32)
    dY = _cpu(dY)
    X = _cpu(X)
    if dY.dtype != X.dtype or dY.dim() != 2 or X.dim() != 2 or dY.shape[0] != X.shape[0]:
        raise ValueError("dY and X must be 2-D, same dtype and batch rows")
    nnzb = ci.numel()
    dw = torch.empty(nnzb, bm, bk, dtype=torch.float32)
    rc = load().oracle_bsr_sddmm(rp.data_ptr(), ci.data_ptr(), rp.numel() - 1, nnzb, dY.data_ptr(), dY.stride(0),
                                 X.data_ptr(), X.stride(0), _DT[dY.dtype], dY.shape[0], dY.shape[1], X.shape[1], bm,
                                 bk, dw.data_ptr(), nthreads)
    if rc:
        raise ValueError(f"oracle_bsr_sddmm failed ({rc})")
    return dw


def bsr_transpose(row_ptr: torch.Tensor, col_idx: torch.Tensor, nbc: int):
    """(row_ptr_t, col_idx_t, perm_t) of W^T, int32."""
    rp = _cpu(row_ptr, torch.int32)
    ci = _cpu(col_idx, torch.int32)
    rpt = torch.empty(nbc + 1, dtype=torch.int32)
    cit = torch.empty(ci.numel(), dtype=torch.int32)
    pt = torch.empty(ci.numel(), dtype=torch.int32)
    rc = load().oracle_bsr_transpose(rp.data_ptr(), ci.data_ptr(), rp.numel() - 1, nbc, rpt.data_ptr(),
                                     cit.data_ptr(), pt.data_ptr())
    if rc:
        raise ValueError("oracle_bsr_transpose: block-column out of range")
    return rpt, cit, pt


def sparse_gather(weight: torch.Tensor, row_offsets: torch.Tensor, mask_cols: torch.Tensor,
                  ids: torch.Tensor) -> torch.Tensor:
    """(len(ids), D) rows of weight on the row's active columns, 0 elsewhere
    and for ids outside [0, N); weight's dtype, bit-exact copies."""
    w = _cpu(weight)
    ro = _cpu(row_offsets, torch.int64)
    mc = _cpu(mask_cols, torch.int64)
    i = _cpu(ids, torch.int64)
    n, d = w.shape
    if ro.numel() < n + 1:
        raise ValueError("row_offsets must hold N + 1 entries")
    out = torch.empty(i.numel(), d, dtype=w.dtype)
    load().oracle_sparse_gather(w.data_ptr(), _DT[w.dtype], n, d, ro.data_ptr(), mc.data_ptr(), i.data_ptr(),
                                i.numel(), out.data_ptr())
    return out


def sparse_scatter_grad(grad_output: torch.Tensor, active_ids: torch.Tensor, batch_ids: torch.Tensor,
                        num_embeddings: int, embedding_dim: int) -> torch.Tensor:
    """(N, D) fp32 gradient: active rows hold the batch-ordered fp32 sum of
    their grad_output rows, every other row is 0."""
    g = _cpu(grad_output)
    a = _cpu(active_ids, torch.int64)
    b = _cpu(batch_ids, torch.int64)
    if g.numel() != b.numel() * embedding_dim:
        raise ValueError("grad_output must be (B, D)")
    out = torch.empty(num_embeddings, embedding_dim, dtype=torch.float32)
    rc = load().oracle_sparse_scatter_grad(g.data_ptr(), _DT[g.dtype], a.data_ptr(), a.numel(), b.data_ptr(),
                                           b.numel(), num_embeddings, embedding_dim, out.data_ptr())
    if rc:
        raise ValueError(f"oracle_sparse_scatter_grad failed ({rc})")
    return out
