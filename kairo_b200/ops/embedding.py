"""Masked embedding lookup and its gradient scatter (CUDA only).

Mirrors the reference's ``kairo.ops.sparse_embedding`` (kairo/ops/
sparse_embedding.py:59-161) on this package's kernels:

* ``sparse_gather(weight, mask, ids)`` -- ``weight[ids]`` with the columns
  that ``mask`` leaves inactive set to zero (sparse_embedding.py:59-101).
  The mask's stable row sort and row offsets (``_sort_coo_by_row`` :49-56,
  ``_coo_to_row_offsets`` :23-46) run on the device (``kairo_coo_sort_rows``)
  once per mask object and are cached; ``sort_mask_rows`` exposes them.
* ``sparse_scatter_grad(grad_output, active_ids, batch_ids, N, D)`` -- the
  (N, D) gradient with the rows of ``active_ids`` holding the sum of their
  batch rows (sparse_embedding.py:104-161), deterministic (fp32 sums in batch
  order, no atomics).

Results are those of the reference's CUDA kernels (csrc/
sparse_embedding_kernel.cu): the mask's values are not read (an entry means
"active") and an id outside [0, N) gathers a zero row.  weight/grad_output
may be float32 (the reference's only dtype), float16 or bfloat16.
"""

from __future__ import annotations

import ctypes
import threading
import weakref
from dataclasses import dataclass

import torch
from torch import Tensor

from kairo_b200 import _lib
from kairo_b200.ops.spmm import _require_cuda
from kairo_b200.types import SparseMask


@dataclass(frozen=True)
class MaskRows:
    """A COO element mask in row order (the reference's CSR view of it).

    row_offsets: (N + 1,) int64; rows/cols: (nnz,) int64 sorted stably by
    row; perm: (nnz,) int64, the mask position of every sorted entry;
    bits: (N, ceil(D / 32)) int32 words, bit c % 32 of word c / 32 set for
    an active (row, c) -- what the gather kernel reads."""

    row_offsets: Tensor
    rows: Tensor
    cols: Tensor
    perm: Tensor
    bits: Tensor
    dense_shape: tuple[int, int]

    @property
    def nnz(self) -> int:
        return int(self.cols.numel())


def _scratch(nbytes: int, device: torch.device) -> Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def sort_mask_rows(mask: SparseMask, device: torch.device | str | None = None, *, check: bool = True) -> MaskRows:
    """Stable sort of ``mask``'s entries by row and the row offsets, on the
    device.  ``check`` synchronises and raises KairoDeviceError when an entry
    lies outside ``dense_shape``."""
    dev = torch.device(device) if device is not None else mask.indices.device
    if dev.type != "cuda":
        raise RuntimeError("kairo_b200.sort_mask_rows runs on CUDA tensors only; this package has no CPU "
                           "implementation")
    n_rows, n_cols = (int(v) for v in mask.dense_shape)
    idx = mask.indices.to(device=dev, dtype=torch.int64)
    if idx.dim() != 2 or idx.shape[0] != 2:
        raise ValueError("mask.indices must be (2, nnz)")
    rows = idx[0].contiguous()
    cols = idx[1].contiguous()
    nnz = rows.numel()
    lib = _lib.lib()
    row_offsets = torch.empty(n_rows + 1, dtype=torch.int64, device=dev)
    rows_s = torch.empty(nnz, dtype=torch.int64, device=dev)
    cols_s = torch.empty(nnz, dtype=torch.int64, device=dev)
    perm = torch.empty(nnz, dtype=torch.int64, device=dev)
    with torch.cuda.device(dev):
        nbytes = ctypes.c_size_t(0)
        _lib.check(lib.kairo_coo_sort_rows_workspace_size(n_rows, nnz, ctypes.byref(nbytes)), "sort_mask_rows")
        ws = _scratch(nbytes.value, dev)
        _lib.check(lib.kairo_coo_sort_rows(_lib.ptr(rows) if nnz else None, _lib.ptr(cols) if nnz else None, nnz,
                                           n_rows, n_cols, row_offsets.data_ptr(),
                                           _lib.ptr(rows_s) if nnz else None, _lib.ptr(cols_s) if nnz else None,
                                           _lib.ptr(perm) if nnz else None, ws.data_ptr(), ws.numel(),
                                           _lib.stream_handle(dev)), "sort_mask_rows")
        if check:
            _lib.raise_on_device_error(ws)
        bits = torch.empty(n_rows, (n_cols + 31) // 32, dtype=torch.int32, device=dev)
        _lib.check(lib.kairo_mask_bits(_lib.ptr(rows) if nnz else None, _lib.ptr(cols) if nnz else None, nnz, n_rows,
                                       n_cols, bits.data_ptr() if bits.numel() else None, _lib.stream_handle(dev)),
                   "sort_mask_rows")
    return MaskRows(row_offsets=row_offsets, rows=rows_s, cols=cols_s, perm=perm, bits=bits,
                    dense_shape=(n_rows, n_cols))


# Row-sorted view of every SparseMask object used with sparse_gather, per
# device, dropped when the mask object is collected.
_cache_lock = threading.Lock()
_mask_cache: dict[int, dict[torch.device, MaskRows]] = {}


def _mask_rows_cached(mask: SparseMask, device: torch.device) -> MaskRows:
    key = id(mask)
    with _cache_lock:
        entry = _mask_cache.get(key)
        if entry is not None and device in entry:
            return entry[device]
    rows = sort_mask_rows(mask, device)
    with _cache_lock:
        if key not in _mask_cache:
            _mask_cache[key] = {}
            weakref.finalize(mask, _mask_cache.pop, key, None)
        _mask_cache[key][device] = rows
    return rows


def _gather(weight: Tensor, mr: MaskRows, ids: Tensor) -> Tensor:
    n, d = weight.shape
    out = torch.empty(ids.numel(), d, dtype=weight.dtype, device=weight.device)
    if ids.numel() == 0:
        return out
    with torch.cuda.device(weight.device):
        _lib.check(_lib.lib().kairo_sparse_gather_bits(weight.data_ptr(), n, d, _lib.kairo_dtype(weight.dtype),
                                                       mr.bits.data_ptr(), ids.data_ptr(), ids.numel(),
                                                       out.data_ptr(), _lib.stream_handle(weight.device)),
                   "sparse_gather")
    return out


def sparse_gather(weight: Tensor, mask: SparseMask | MaskRows, ids: Tensor) -> Tensor:
    """Masked embedding lookup: (len(ids), D) rows of ``weight`` with the
    columns inactive in ``mask`` zeroed (kairo/ops/sparse_embedding.py:59-101).

    ``mask`` is a SparseMask over (N, D) or its ``sort_mask_rows`` view."""
    _require_cuda(weight, op="sparse_gather")
    if weight.dim() != 2:
        raise ValueError("weight must be 2-D (N, D)")
    if ids.numel() == 0:
        return torch.zeros(0, weight.shape[1], dtype=weight.dtype, device=weight.device)
    mr = mask if isinstance(mask, MaskRows) else _mask_rows_cached(mask, weight.device)
    if tuple(mr.dense_shape) != tuple(weight.shape):
        raise ValueError(f"the mask is {tuple(mr.dense_shape)}; weight is {tuple(weight.shape)}")
    ids = ids.to(device=weight.device, dtype=torch.int64).reshape(-1).contiguous()
    return _gather(weight.contiguous(), mr, ids)


def sparse_scatter_grad(grad_output: Tensor, active_ids: Tensor, batch_ids: Tensor, num_embeddings: int,
                        embedding_dim: int, *, check: bool = False) -> Tensor:
    """(num_embeddings, embedding_dim) gradient: row r of ``active_ids``
    (sorted, unique) holds the sum of ``grad_output[b]`` over ``batch_ids[b]
    == r``; every other row is zero (kairo/ops/sparse_embedding.py:104-161).

    ``check=True`` synchronises and raises KairoDeviceError on an active id
    outside [0, num_embeddings)."""
    _require_cuda(grad_output, op="sparse_scatter_grad")
    n, d = int(num_embeddings), int(embedding_dim)
    dev = grad_output.device
    if active_ids.numel() == 0 or batch_ids.numel() == 0:
        return torch.zeros(n, d, dtype=grad_output.dtype, device=dev)
    if n <= 0 or d <= 0:
        raise ValueError("num_embeddings and embedding_dim must be positive")
    if grad_output.dim() != 2 or grad_output.shape[0] != batch_ids.numel() or grad_output.shape[1] != d:
        raise ValueError(f"grad_output must be ({batch_ids.numel()}, {d}), got {tuple(grad_output.shape)}")
    g = grad_output.contiguous()
    aid = active_ids.to(device=dev, dtype=torch.int64).reshape(-1).contiguous()
    bid = batch_ids.to(device=dev, dtype=torch.int64).reshape(-1).contiguous()
    out = torch.empty(n, d, dtype=g.dtype, device=dev)
    lib = _lib.lib()
    with torch.cuda.device(dev):
        nbytes = ctypes.c_size_t(0)
        _lib.check(lib.kairo_sparse_scatter_grad_workspace_size(aid.numel(), bid.numel(), ctypes.byref(nbytes)),
                   "sparse_scatter_grad")
        ws = _scratch(nbytes.value, dev)
        _lib.check(lib.kairo_sparse_scatter_grad(g.data_ptr(), _lib.kairo_dtype(g.dtype), aid.data_ptr(), aid.numel(),
                                                 bid.data_ptr(), bid.numel(), n, d, out.data_ptr(), ws.data_ptr(),
                                                 ws.numel(), _lib.stream_handle(dev)), "sparse_scatter_grad")
        if check:
            _lib.raise_on_device_error(ws)
    return out
