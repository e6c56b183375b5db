"""Masked embedding gather / gradient scatter on the GPU against the golden
fixtures (made from the reference's own code) and the CPU oracle.

Bit-exact throughout: the mask sort and row offsets are integer work, the
gather copies elements, and the scatter sums fp32 in batch order exactly as
the oracle (and the reference's index_add_) does; 2-byte results are the
oracle's fp32 sums rounded once.
"""

from __future__ import annotations

from pathlib import Path

import pytest
import torch

from oracle import oracle
from kairo_b200 import _C, _lib
from kairo_b200.ops import sort_mask_rows, sparse_gather, sparse_scatter_grad
from kairo_b200.types import SparseMask

pytestmark = pytest.mark.gpu

DEV = "cuda"
HERE = Path(__file__).parent / "golden"
GATHER = sorted(HERE.glob("emb_*gather*.pt"))
SCATTER = sorted(HERE.glob("emb_*scatter*.pt"))


def _load(path):
    return torch.load(path, weights_only=False)


def _mask(g, device=DEV):
    return SparseMask(indices=g["mask_indices"].to(device), values=torch.ones(g["mask_indices"].shape[1], device=device),
                      dense_shape=g["mask_shape"], sparsity_ratio=0.0)


def _bits(t):
    t = t.cpu()
    return t.view(torch.int16) if t.element_size() == 2 else t.view(torch.int32)


@pytest.mark.parametrize("path", GATHER, ids=lambda p: p.stem)
def test_mask_sort_vs_golden(path):
    g = _load(path)
    mr = sort_mask_rows(_mask(g))
    assert torch.equal(mr.row_offsets.cpu(), g["row_offsets"])
    assert torch.equal(mr.rows.cpu(), g["rows_sorted"])
    assert torch.equal(mr.cols.cpu(), g["cols_sorted"])
    assert torch.equal(mr.perm.cpu(), g["perm"])


@pytest.mark.parametrize("path", GATHER, ids=lambda p: p.stem)
def test_gather_vs_golden(path):
    g = _load(path)
    w = g["weight"].to(DEV)
    m = _mask(g)
    for ids, out in zip(g["ids"], g["out"]):
        got = sparse_gather(w, m, ids.to(DEV))
        assert got.shape == out.shape and got.dtype == out.dtype
        assert torch.equal(got.cpu(), out)
        # the reference's extension entry point, on the reference's own inputs
        got2 = _C.sparse_gather_forward(w, g["rows_sorted"].to(DEV), g["cols_sorted"].to(DEV), ids.to(DEV),
                                        g["row_offsets"].to(DEV))
        assert torch.equal(got2.cpu(), out)


@pytest.mark.parametrize("path", SCATTER, ids=lambda p: p.stem)
def test_scatter_vs_golden(path):
    g = _load(path)
    got = sparse_scatter_grad(g["grad_output"].to(DEV), g["active_ids"].to(DEV), g["batch_ids"].to(DEV), g["N"],
                              g["D"], check=True)
    assert torch.equal(got.cpu(), g["grad_weight"])
    got2 = _C.sparse_scatter_backward(g["grad_output"].to(DEV), g["active_ids"].to(DEV), g["batch_ids"].to(DEV),
                                      g["N"], g["D"])
    assert torch.equal(got2.cpu(), g["grad_weight"])


def _random_mask(n, d, density, seed, shuffle=True):
    gen = torch.Generator().manual_seed(seed)
    keep = torch.rand(n, d, generator=gen) < density
    r, c = keep.nonzero(as_tuple=True)
    if shuffle:
        p = torch.randperm(r.numel(), generator=gen)
        r, c = r[p], c[p]
    return SparseMask(indices=torch.stack([r, c]), values=torch.ones(r.numel()), dense_shape=(n, d),
                      sparsity_ratio=1.0 - r.numel() / (n * d))


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape", [(1000, 64, 0.2, 4096), (5000, 300, 0.05, 1000), (64, 5000, 0.6, 129),
                                   (3000, 96, 0.3, 20001)])   # a large batch: 32 ids per warp
def test_gather_vs_oracle(dtype, shape):
    n, d, density, b = shape
    m = _random_mask(n, d, density, seed=n + d)
    w = torch.randn(n, d).to(dtype)
    gen = torch.Generator().manual_seed(3)
    ids = torch.randint(-3, n + 3, (b,), generator=gen)  # a few out of range: zero rows
    mr = sort_mask_rows(m, DEV)
    perm, rs, cs = oracle.sort_coo_by_row(m.indices[0], m.indices[1], n)
    assert torch.equal(mr.row_offsets.cpu(), oracle.row_offsets(rs, n))
    assert torch.equal(mr.cols.cpu(), cs) and torch.equal(mr.perm.cpu(), perm)
    got = sparse_gather(w.to(DEV), mr, ids.to(DEV))
    exp = oracle.sparse_gather(w, oracle.row_offsets(rs, n), cs, ids)
    assert got.dtype == dtype
    assert torch.equal(_bits(got), _bits(exp))
    # the row-offset kernel behind the reference's extension entry point
    got_csr = _C.sparse_gather_forward(w.to(DEV), mr.rows, mr.cols, ids.to(DEV), mr.row_offsets)
    assert torch.equal(_bits(got_csr), _bits(exp))
    # a weight that is not 16-byte aligned takes the scalar path
    flat = torch.empty(n * d + 1, dtype=dtype, device=DEV)
    wm = flat[1:].view(n, d)
    wm.copy_(w.to(DEV))
    assert torch.equal(_bits(sparse_gather(wm, mr, ids.to(DEV))), _bits(exp))


def test_gather_long_rows_and_cache():
    """Rows of more than 16384 entries (kept in scatter order by the device
    sort) gather the same values; a SparseMask's row view is cached."""
    n, d = 6, 20000
    m = _random_mask(n, d, 0.95, seed=5)
    w = torch.randn(n, d)
    ids = torch.tensor([5, 0, 3, 3, 1])
    mr = sort_mask_rows(m, DEV)
    _, rs, cs = oracle.sort_coo_by_row(m.indices[0], m.indices[1], n)
    ro = oracle.row_offsets(rs, n)
    assert torch.equal(mr.row_offsets.cpu(), ro)
    # each row holds the same set of columns
    for r in range(n):
        a, b = int(ro[r]), int(ro[r + 1])
        assert torch.equal(torch.sort(mr.cols.cpu()[a:b]).values, torch.sort(cs[a:b]).values)
    got = sparse_gather(w.to(DEV), m, ids.to(DEV))
    assert torch.equal(got.cpu(), oracle.sparse_gather(w, ro, cs, ids))
    again = sparse_gather(w.to(DEV), m, ids.to(DEV))
    assert torch.equal(got, again)


def test_gather_edge_cases():
    w = torch.randn(10, 8, device=DEV)
    m = _random_mask(10, 8, 0.5, seed=1)
    assert sparse_gather(w, m, torch.tensor([], dtype=torch.int64, device=DEV)).shape == (0, 8)
    empty = SparseMask(indices=torch.zeros(2, 0, dtype=torch.int64), values=torch.zeros(0), dense_shape=(10, 8),
                       sparsity_ratio=1.0)
    out = sparse_gather(w, empty, torch.tensor([0, 1, 9], device=DEV))
    assert out.shape == (3, 8) and int(out.abs().sum()) == 0
    bad = SparseMask(indices=torch.tensor([[0, 10], [1, 2]]), values=torch.ones(2), dense_shape=(10, 8),
                     sparsity_ratio=0.0)
    with pytest.raises(_lib.KairoDeviceError):
        sort_mask_rows(bad, DEV)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("case", [
    # n, d, batch, hot share: the hottest id's share of the batch
    (1000, 64, 4096, 0.0),
    (20000, 200, 3000, 0.0),
    (300, 16, 40000, 0.6),      # one row with > 16384 members: summed by an in-order batch scan
    (50, 1, 100, 0.0),          # D = 1
])
def test_scatter_vs_oracle(dtype, case):
    n, d, b, hot = case
    gen = torch.Generator().manual_seed(n + b)
    batch = torch.randint(0, n, (b,), generator=gen)
    if hot:
        batch[torch.rand(b, generator=gen) < hot] = 7
    active = torch.unique(torch.cat([torch.unique(batch)[::2], torch.tensor([7])]))
    grad = torch.randn(b, d, generator=gen).to(dtype)
    got = sparse_scatter_grad(grad.to(DEV), active.to(DEV), batch.to(DEV), n, d, check=True)
    exp = oracle.sparse_scatter_grad(grad, active, batch, n, d)
    assert got.dtype == dtype
    assert torch.equal(_bits(got), _bits(exp.to(dtype)))


def test_scatter_mostly_inactive_batch():
    # Nearly every batch position names an inactive row: they all share the
    # bucket after the active ones, one longer than the shared-memory sort
    # takes, which the sums must ignore.
    gen = torch.Generator().manual_seed(12)
    n, d, b = 100000, 32, 50000
    batch = torch.randint(0, n, (b,), generator=gen)
    active = torch.unique(batch[:3])
    grad = torch.randn(b, d, generator=gen)
    got = sparse_scatter_grad(grad.to(DEV), active.to(DEV), batch.to(DEV), n, d, check=True)
    assert torch.equal(got.cpu(), oracle.sparse_scatter_grad(grad, active, batch, n, d))


def test_scatter_edge_cases():
    g = torch.randn(3, 4, device=DEV)
    e = torch.tensor([], dtype=torch.int64, device=DEV)
    assert int(sparse_scatter_grad(g, e, torch.tensor([0, 1, 2], device=DEV), 5, 4).abs().sum()) == 0
    assert int(sparse_scatter_grad(torch.zeros(0, 4, device=DEV), torch.tensor([0, 1], device=DEV), e, 5,
                                   4).abs().sum()) == 0
    # an active id with no batch member, duplicated active ids counted once
    got = sparse_scatter_grad(g, torch.tensor([1, 1, 4], device=DEV), torch.tensor([1, 2, 1], device=DEV), 5, 4)
    exp = torch.zeros(5, 4)
    exp[1] = g[0].cpu() + g[2].cpu()
    assert torch.equal(got.cpu(), exp)
    with pytest.raises(_lib.KairoDeviceError):
        sparse_scatter_grad(g, torch.tensor([1, 9], device=DEV), torch.tensor([9, 1, 1], device=DEV), 5, 4,
                            check=True)
