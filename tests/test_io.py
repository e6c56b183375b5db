"""On-disk BSR format: round trip and validation (CPU)."""

from __future__ import annotations

import pytest
import torch

from kairo_b200.io import load_bsr, save_bsr
from kairo_b200.types import BlockSparseMatrix


def _matrix(shuffled: bool):
    g = torch.Generator().manual_seed(0)
    rp = torch.tensor([0, 2, 2, 5], dtype=torch.int32)
    ci = torch.tensor([0, 3, 1, 2, 3], dtype=torch.int32)
    blocks = torch.randn(5, 16, 16, generator=g).to(torch.bfloat16)
    if not shuffled:
        return BlockSparseMatrix(rp, ci, blocks, (40, 64), (16, 16))
    blk = torch.tensor([4, 2, 0, 3, 1], dtype=torch.int32)
    return BlockSparseMatrix(rp, ci, blocks, (40, 64), (16, 16), blk_idx=blk)


@pytest.mark.parametrize("shuffled", [False, True])
def test_round_trip(tmp_path, shuffled):
    a = _matrix(shuffled)
    path = tmp_path / "w.kbsr"
    save_bsr(a, path)
    b = load_bsr(path)
    assert b.shape == a.shape and b.block_size == a.block_size and b.blk_idx is None
    assert torch.equal(b.row_ptr, a.row_ptr) and torch.equal(b.col_idx, a.col_idx)
    want = a.blocks if a.blk_idx is None else a.blocks[a.blk_idx.long()]
    assert torch.equal(b.blocks, want)
    assert b.max_row_blocks == 3
    d = torch.load(path, weights_only=True)
    assert d["row_ptr"].dtype == torch.int64 and d["format"] == "kairo-bsr"


def test_rejects_bad_files(tmp_path):
    p = tmp_path / "x.pt"
    torch.save({"format": "other"}, p)
    with pytest.raises(ValueError):
        load_bsr(p)
    a = _matrix(False)
    save_bsr(a, p)
    d = torch.load(p, weights_only=True)
    d["col_idx"] = torch.tensor([0, 3, 1, 2, 9], dtype=torch.int32)  # past the 4 block-columns
    torch.save(d, p)
    with pytest.raises(ValueError, match="block grid"):
        load_bsr(p)
    d["col_idx"] = a.col_idx
    d["row_ptr"] = torch.tensor([0, 3, 2, 5])
    torch.save(d, p)
    with pytest.raises(ValueError, match="monotone"):
        load_bsr(p)
