"""On-disk format of a BlockSparseMatrix.

The reference has no sparse-matrix file format (``SparseMask``'s COO lists are
its only interchange type, kairo/types.py:10-40).  This one is a ``torch.save``
dict, so it needs nothing beyond PyTorch to read:

    format          "kairo-bsr"
    version         1
    shape           (M, K)
    block_size      (bm, bk)
    row_ptr         (nbr + 1,) int64  -- the reference's row-offset convention
                                         (kairo/ops/sparse_embedding.py:23-46)
    col_idx         (nnzb,) int32
    blocks          (nnzb, bm, bk)    -- in BSR order (any blk_idx applied)
    max_row_blocks  int               -- longest block-row

``save_bsr`` writes from any device; ``load_bsr`` validates the structure on
the CPU (monotone offsets, ids inside the block grid) before placing the
tensors on the requested device.
"""

from __future__ import annotations

import os
from typing import Any

import torch

from kairo_b200.types import BlockSparseMatrix

FORMAT = "kairo-bsr"
VERSION = 1


def _to_payload(a: BlockSparseMatrix) -> dict[str, Any]:
    blocks = a.blocks if a.blk_idx is None else a.blocks[a.blk_idx.long()]
    rp = a.row_ptr.detach().to("cpu", torch.int64)
    longest = int((rp[1:] - rp[:-1]).max()) if rp.numel() > 1 else 0
    return {
        "format": FORMAT,
        "version": VERSION,
        "shape": tuple(int(v) for v in a.shape),
        "block_size": tuple(int(v) for v in a.block_size),
        "row_ptr": rp.contiguous(),
        "col_idx": a.col_idx.detach().to("cpu", torch.int32).contiguous(),
        "blocks": blocks.detach().to("cpu").contiguous(),
        "max_row_blocks": longest,
    }


def save_bsr(a: BlockSparseMatrix, path: str | os.PathLike) -> None:
    """Write ``a`` to ``path`` (atomically: a temporary file is renamed)."""
    tmp = f"{os.fspath(path)}.tmp"
    torch.save(_to_payload(a), tmp)
    os.replace(tmp, path)


def load_bsr(path: str | os.PathLike, device: str | torch.device = "cpu") -> BlockSparseMatrix:
    """Read a file written by ``save_bsr``; raises ValueError if it is not a
    valid kairo-bsr file."""
    d = torch.load(path, map_location="cpu", weights_only=True)
    if not isinstance(d, dict) or d.get("format") != FORMAT:
        raise ValueError(f"{path}: not a {FORMAT} file")
    if d.get("version") != VERSION:
        raise ValueError(f"{path}: unsupported {FORMAT} version {d.get('version')!r}")
    m, k = (int(v) for v in d["shape"])
    bm, bk = (int(v) for v in d["block_size"])
    rp = torch.as_tensor(d["row_ptr"], dtype=torch.int64)
    ci = torch.as_tensor(d["col_idx"], dtype=torch.int32)
    blocks = d["blocks"]
    nbr = (m + bm - 1) // bm
    nbc = (k + bk - 1) // bk
    if rp.dim() != 1 or rp.numel() != nbr + 1 or int(rp[0]) != 0 or int(rp[-1]) != ci.numel():
        raise ValueError(f"{path}: row_ptr does not match the shape and block count")
    if rp.numel() > 1 and bool((rp[1:] < rp[:-1]).any()):
        raise ValueError(f"{path}: row_ptr is not monotone")
    if ci.numel() and (int(ci.min()) < 0 or int(ci.max()) >= nbc):
        raise ValueError(f"{path}: block-column id outside the block grid")
    if blocks.dim() != 3 or tuple(blocks.shape) != (ci.numel(), bm, bk):
        raise ValueError(f"{path}: blocks must be ({ci.numel()}, {bm}, {bk})")
    dev = torch.device(device)
    return BlockSparseMatrix(row_ptr=rp.to(torch.int32).to(dev), col_idx=ci.to(dev), blocks=blocks.to(dev),
                             shape=(m, k), block_size=(bm, bk), max_row_blocks=int(d.get("max_row_blocks", 0)))
