"""CPU checks of the oracle's backward restatements (no GPU needed).

The reference has no SpMM backward, so these oracle functions are pinned to
their definitions instead of reference fixtures: the transpose to a stable
sort of W's positions by block-column, the SDDMM to float64 products of the
dense slices.
"""

from __future__ import annotations

import numpy as np
import torch

from oracle import oracle


def _random_bsr(nbr, nbc, density, seed):
    g = torch.Generator().manual_seed(seed)
    mask = torch.rand(nbr, nbc, generator=g) < density
    rows, cols = mask.nonzero(as_tuple=True)
    counts = torch.bincount(rows, minlength=nbr)
    row_ptr = torch.zeros(nbr + 1, dtype=torch.int32)
    row_ptr[1:] = torch.cumsum(counts, 0)
    return row_ptr, cols.to(torch.int32), rows


def test_transpose_is_stable_sort_by_column():
    for seed, (nbr, nbc, d) in enumerate([(5, 7, 0.4), (40, 13, 0.2), (1, 9, 1.0), (6, 1, 0.5), (4, 4, 0.0)]):
        rp, ci, rows = _random_bsr(nbr, nbc, d, seed)
        rpt, cit, pt = oracle.bsr_transpose(rp, ci, nbc)
        order = np.argsort(ci.numpy(), kind="stable")
        assert np.array_equal(pt.numpy(), order)
        assert np.array_equal(cit.numpy(), rows.numpy()[order])
        assert np.array_equal(rpt.numpy(), np.concatenate([[0], np.cumsum(np.bincount(ci.numpy(), minlength=nbc))]))


def test_sddmm_matches_float64_slices():
    for seed, (nbr, nbc, bs, n, dt) in enumerate([(3, 4, 4, 7, torch.float32), (5, 3, 16, 33, torch.float16),
                                                   (2, 6, 8, 64, torch.bfloat16)]):
        rp, ci, rows = _random_bsr(nbr, nbc, 0.5, seed)
        g = torch.Generator().manual_seed(100 + seed)
        dy = torch.randn(n, nbr * bs, generator=g).to(dt)
        x = torch.randn(n, nbc * bs, generator=g).to(dt)
        dw = oracle.bsr_sddmm(rp, ci, dy, x, bs, bs)
        for p in range(ci.numel()):
            i, j = int(rows[p]), int(ci[p])
            ref = dy[:, i * bs:(i + 1) * bs].double().T @ x[:, j * bs:(j + 1) * bs].double()
            assert torch.allclose(dw[p].double(), ref, rtol=1e-5, atol=1e-4 * (1 + ref.abs().max()))
