"""Block pruning on the device against the reference's selection rules.

The reference's element-level rules (kairo/training/sparse_rec/topology.py)
are applied to block scores on the CPU (torch.topk + sort for pruning,
"active = -1" + topk for growth) and compared with the device path: block
norms within fp32 rounding of float64, selected index sets bit-exact.
"""

from __future__ import annotations

import pytest
import torch

from kairo_b200.ops import bsr_from_tiles
from kairo_b200.pruning import (
    block_magnitude_mask,
    block_norms,
    bsr_block_norms,
    grow_blocks,
    prune_blocks,
    topk_indices,
    update_blocks,
)
from kairo_b200.workloads import WorkloadSpec, generate

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("shape", [(256, 512, 64), (100, 70, 16), (1024, 2048, 32)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_block_norms(shape, dtype):
    m, k, bs = shape
    g = torch.Generator().manual_seed(1)
    a = torch.randn(m, k, generator=g).to(dtype)
    n = block_norms(a.to(DEV), bs).cpu().double()
    nbr, nbc = (m + bs - 1) // bs, (k + bs - 1) // bs
    pad = torch.zeros(nbr * bs, nbc * bs, dtype=torch.float64)
    pad[:m, :k] = a.double()
    ref = pad.view(nbr, bs, nbc, bs).pow(2).sum(dim=(1, 3)).sqrt()
    assert torch.allclose(n, ref, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("n,count", [(1, 1), (1000, 1), (1000, 999), (65536, 13107), (1 << 20, 5000)])
def test_topk_indices_matches_sorted_topk(n, count):
    g = torch.Generator().manual_seed(n + count)
    s = torch.randn(n, generator=g)
    got = topk_indices(s.to(DEV), count).cpu()
    ref = s.topk(count).indices.sort().values
    assert torch.equal(got, ref)


def test_topk_indices_ties_and_nan():
    s = torch.tensor([1.0, 3.0, 3.0, float("nan"), 3.0, -2.0, 0.0, 3.0])
    # threshold 3.0 is shared by four entries; two are needed -> the two lowest indices
    assert topk_indices(s.to(DEV), 2).cpu().tolist() == [1, 2]
    # all four 3.0 entries plus the 1.0, listed in index order
    assert topk_indices(s.to(DEV), 5).cpu().tolist() == [0, 1, 2, 4, 7]
    assert topk_indices(s.to(DEV), 8).cpu().tolist() == list(range(8))  # NaN taken last, still listed in order
    assert topk_indices(torch.tensor([-0.0, 0.0, -1.0]).to(DEV), 2).cpu().tolist() == [0, 1]


def _ref_topk_ties(s: torch.Tensor, count: int) -> torch.Tensor:
    """Indices of the `count` largest scores, ties to the lower index, NaN
    lowest, -0.0 below +0.0 (the kernels' order-preserving key), ascending."""
    import numpy as np

    b = s.numpy().view(np.uint32)
    key = np.where(b & 0x80000000, ~b, b | 0x80000000).astype(np.uint64)
    key[np.isnan(s.numpy())] = 0
    order = np.lexsort((np.arange(len(b)), -key.astype(np.int64)))
    return torch.from_numpy(np.sort(order[:count]).astype(np.int64))


@pytest.mark.parametrize("n", [5000, 1 << 18, 300000])
def test_topk_indices_ties_quantised(n):
    """Quantised scores (many ties at every threshold) and NaNs."""
    g = torch.Generator().manual_seed(n)
    s = torch.randint(-20, 20, (n,), generator=g).float() / 4
    s[torch.randint(0, n, (n // 100,), generator=g)] = float("nan")
    for count in (1, n // 7, n // 2, n - 3):
        got = topk_indices(s.to(DEV), count).cpu()
        assert torch.equal(got, _ref_topk_ties(s, count))


def test_block_magnitude_mask_matches_reference_rule():
    g = torch.Generator().manual_seed(7)
    w = (torch.randn(1024, 4096, generator=g) * 0.02).to(torch.bfloat16)
    mask = block_magnitude_mask(w.to(DEV), 64, 0.2)
    norms = block_norms(w.to(DEV), 64).cpu().reshape(-1)
    keep = int(norms.numel() * 0.2)
    ref = norms.topk(keep).indices.sort().values
    nbc = 4096 // 64
    got = (mask.indices[0] * nbc + mask.indices[1]).cpu()
    assert torch.equal(got, ref)
    assert mask.dense_shape == (1024 // 64, nbc) and mask.nnz == keep


def _weight(seed):
    spec = WorkloadSpec("w", torch.bfloat16, 512, 1024, 8, 32, 0.8, a_std=0.1)
    p = generate(spec, seed=seed)
    return bsr_from_tiles(p.tiles.to(DEV), p.row_ids.to(DEV), p.col_ids.to(DEV), (512, 1024))


def test_prune_blocks_reference_rule():
    w = _weight(3)
    norms = bsr_block_norms(w).cpu()
    pruned = prune_blocks(w, 0.3)
    keep = w.nnzb - int(w.nnzb * 0.3)
    pos = norms.topk(keep).indices.sort().values
    assert pruned.nnzb == keep
    assert torch.equal(pruned.col_idx.cpu(), w.col_idx.cpu()[pos])
    assert torch.equal(pruned.blocks.cpu(), w.blocks.cpu()[pos])
    rows = torch.repeat_interleave(torch.arange(w.nbr), (w.row_ptr[1:] - w.row_ptr[:-1]).cpu().long())[pos]
    assert torch.equal(pruned.row_ptr.cpu()[1:], torch.cumsum(torch.bincount(rows, minlength=w.nbr), 0).int())


def test_grow_and_update_blocks():
    w = _weight(4)
    g = torch.Generator().manual_seed(5)
    scores = torch.rand(w.nbr, w.nbc, generator=g)
    grown = grow_blocks(w, scores.to(DEV), 40)
    # the reference rule on the CPU: active positions score -1, take the top 40
    rows = torch.repeat_interleave(torch.arange(w.nbr), (w.row_ptr[1:] - w.row_ptr[:-1]).cpu().long())
    flat = scores.reshape(-1).clone()
    flat[rows * w.nbc + w.col_idx.cpu().long()] = -1.0
    new = set(flat.topk(40).indices.tolist())
    grows = torch.repeat_interleave(torch.arange(w.nbr), (grown.row_ptr[1:] - grown.row_ptr[:-1]).cpu().long())
    got = set((grows * w.nbc + grown.col_idx.cpu().long()).tolist())
    old = set((rows * w.nbc + w.col_idx.cpu().long()).tolist())
    assert got == old | new and grown.nnzb == w.nnzb + 40
    assert torch.equal(grown.blocks.float().abs().sum(dim=(1, 2)) == 0,
                       torch.tensor([(int(r) * w.nbc + int(c)) in new for r, c in zip(grows, grown.col_idx.cpu())],
                                    device=DEV))
    res = update_blocks(w, scores.to(DEV), 0.1)
    assert res.num_pruned == int(w.nnzb * 0.1) and res.num_grown == res.num_pruned
    assert res.matrix.nnzb == w.nnzb
