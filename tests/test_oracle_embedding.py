"""Pins the masked-embedding oracle to the reference: the fixtures written by
tests/golden/make_golden_embedding.py from the reference's own code
(kairo/ops/sparse_embedding.py) must be reproduced bit for bit -- the gather
is a copy, the scatter an fp32 sum in batch order on both sides -- and the
reference's unit-test expectations hold for the oracle.  Also covers the
argument checks of the kairo._C-style wrappers, which run before any device
work."""

from __future__ import annotations

from pathlib import Path

import pytest
import torch

from oracle import oracle

HERE = Path(__file__).parent / "golden"
GATHER = sorted(HERE.glob("emb_*gather*.pt"))
SCATTER = sorted(HERE.glob("emb_*scatter*.pt"))


def _load(path: Path) -> dict:
    return torch.load(path, weights_only=False)


def test_fixture_set_present():
    names = {p.stem for p in GATHER + SCATTER}
    assert {"emb_ref_gather", "emb_ref_gather_empty_mask", "emb_unsorted_gather", "emb_ref_scatter",
            "emb_ref_scatter_inactive", "emb_skewed_scatter"} <= names


@pytest.mark.parametrize("path", GATHER, ids=lambda p: p.stem)
def test_oracle_mask_sort_bit_exact(path):
    g = _load(path)
    n = g["mask_shape"][0]
    perm, rs, cs = oracle.sort_coo_by_row(g["mask_indices"][0], g["mask_indices"][1], n)
    assert torch.equal(perm, g["perm"])
    assert torch.equal(rs, g["rows_sorted"]) and torch.equal(cs, g["cols_sorted"])
    assert torch.equal(oracle.row_offsets(rs, n), g["row_offsets"])


@pytest.mark.parametrize("path", GATHER, ids=lambda p: p.stem)
def test_oracle_gather_bit_exact(path):
    g = _load(path)
    for ids, out in zip(g["ids"], g["out"]):
        got = oracle.sparse_gather(g["weight"], g["row_offsets"], g["cols_sorted"], ids)
        assert got.shape == out.shape and got.dtype == out.dtype
        assert torch.equal(got, out)


@pytest.mark.parametrize("path", SCATTER, ids=lambda p: p.stem)
def test_oracle_scatter_bit_exact(path):
    g = _load(path)
    got = oracle.sparse_scatter_grad(g["grad_output"], g["active_ids"], g["batch_ids"], g["N"], g["D"])
    assert torch.equal(got, g["grad_weight"])


def test_oracle_reference_unit_expectations():
    """tests/ops/test_sparse_embedding_ops.py:161-215 of the reference."""
    torch.manual_seed(42)
    grad = torch.randn(4, 8)
    got = oracle.sparse_scatter_grad(grad, torch.tensor([1, 3, 5]), torch.tensor([1, 3, 1, 5]), 10, 8)
    exp = torch.zeros(10, 8)
    exp[1] = grad[0] + grad[2]
    exp[3] = grad[1]
    exp[5] = grad[3]
    assert torch.equal(got, exp)
    assert torch.all(oracle.sparse_scatter_grad(torch.randn(3, 4), torch.tensor([], dtype=torch.int64),
                                                torch.tensor([0, 1, 2]), 5, 4) == 0)
    assert torch.all(oracle.sparse_scatter_grad(torch.zeros(0, 4), torch.tensor([0, 1]),
                                                torch.tensor([], dtype=torch.int64), 5, 4) == 0)


def test_oracle_gather_out_of_range_and_half():
    """Ids outside [0, N) give zero rows (the reference kernels' early return);
    2-byte dtypes are copied bit for bit."""
    w = torch.randn(6, 5).to(torch.bfloat16)
    ro = torch.tensor([0, 5, 5, 7, 7, 8, 8])
    cols = torch.tensor([0, 1, 2, 3, 4, 4, 0, 2])
    got = oracle.sparse_gather(w, ro, cols, torch.tensor([0, -1, 6, 2, 4]))
    exp = torch.zeros(5, 5, dtype=torch.bfloat16)
    exp[0] = w[0]
    exp[3, [4, 0]] = w[2, [4, 0]]
    exp[4, 2] = w[4, 2]
    assert torch.equal(got.view(torch.int16), exp.view(torch.int16))


def test_oracle_scatter_rejects_bad_active_id():
    with pytest.raises(ValueError):
        oracle.sparse_scatter_grad(torch.ones(2, 3), torch.tensor([0, 9]), torch.tensor([0, 1]), 4, 3)


def test_extension_argument_checks():
    """The kairo._C-style wrappers raise the reference's messages
    (csrc/bindings.cpp:46-79) before any device work."""
    from kairo_b200 import _C

    w = torch.randn(8, 6)
    i64 = torch.zeros(4, dtype=torch.int64)
    with pytest.raises(RuntimeError, match="weight must be contiguous"):
        _C.sparse_gather_forward(w.t(), i64, i64, i64, i64)
    with pytest.raises(RuntimeError, match="mask_cols must be int64"):
        _C.sparse_gather_forward(w, i64, i64.int(), i64, i64)
    with pytest.raises(RuntimeError, match="batch_ids must be int64"):
        _C.sparse_gather_forward(w, i64, i64, i64.int(), i64)
    with pytest.raises(RuntimeError, match="weight must be float32"):
        _C.sparse_gather_forward(w.double(), i64, i64, i64, i64)
    with pytest.raises(RuntimeError, match="weight must be on CUDA"):
        _C.sparse_gather_forward(w, i64, i64, i64, torch.zeros(9, dtype=torch.int64))
    g = torch.randn(4, 6)
    with pytest.raises(RuntimeError, match="N must be positive"):
        _C.sparse_scatter_backward(g, i64, i64, 0, 6)
    with pytest.raises(RuntimeError, match="D must be positive"):
        _C.sparse_scatter_backward(g, i64, i64, 5, 0)
    with pytest.raises(RuntimeError, match="active_ids must be int64"):
        _C.sparse_scatter_backward(g, i64.int(), i64, 5, 6)
    with pytest.raises(RuntimeError, match="grad_output must be on CUDA"):
        _C.sparse_scatter_backward(g, i64, i64, 5, 6)
