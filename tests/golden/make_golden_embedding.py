"""Generates the golden fixtures of the masked-embedding path from the reference.

Usage (needs the reference source tree; run where it is mounted):
    python tests/golden/make_golden_embedding.py --ref <path of the reference source tree>

Imports the reference's own ``kairo.ops.sparse_embedding`` (its PyTorch path:
``kairo._C`` is not built, so ``sparse_gather`` / ``sparse_scatter_grad`` run
their fallbacks, kairo/ops/sparse_embedding.py:98-101 and :146-161) and
records, for seeded inputs:
  * _sort_coo_by_row (:49-56) and _coo_to_row_offsets (:23-46) of the mask
  * sparse_gather(weight, mask, ids) for each id list
  * sparse_scatter_grad(grad_output, active_ids, batch_ids, N, D)
The inputs of the reference's unit tests (tests/ops/
test_sparse_embedding_ops.py) are regenerated with the same seeds and draw
order.  Each case is saved as tests/golden/emb_<name>.pt.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent


def _ref(ref: Path):
    sys.path.insert(0, str(ref))
    import kairo.ops.sparse_embedding as se  # noqa: E402
    import kairo.types as ktypes  # noqa: E402

    sys.path.pop(0)
    assert not se.cuda_ext_available(), "the reference extension must be absent: fixtures record the fallback"
    return se, ktypes


def _gather_case(se, name, weight, mask, id_lists):
    rows_s, cols_s = se._sort_coo_by_row(mask)
    out = {"name": name, "torch_version": torch.__version__, "weight": weight.clone(),
           "mask_indices": mask.indices.clone(), "mask_shape": tuple(mask.dense_shape),
           "perm": torch.argsort(mask.indices[0], stable=True), "rows_sorted": rows_s.clone(),
           "cols_sorted": cols_s.clone(), "row_offsets": se._coo_to_row_offsets(rows_s, mask.dense_shape[0]).clone(),
           "ids": [i.clone() for i in id_lists],
           "out": [se.sparse_gather(weight, mask, i).clone() for i in id_lists]}
    torch.save(out, HERE / f"emb_{name}.pt")


def _scatter_case(se, name, grad, active, batch, n, d):
    out = {"name": name, "torch_version": torch.__version__, "grad_output": grad.clone(), "active_ids": active.clone(),
           "batch_ids": batch.clone(), "N": n, "D": d,
           "grad_weight": se.sparse_scatter_grad(grad, active, batch, n, d).clone()}
    torch.save(out, HERE / f"emb_{name}.pt")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of the reference source tree (read-only)")
    args = ap.parse_args()
    se, kt = _ref(Path(args.ref))

    # -- the reference's unit-test inputs (test_sparse_embedding_ops.py:21-55)
    torch.manual_seed(42)
    weight = torch.randn(10, 8)
    torch.manual_seed(42)
    n, d = 10, 8
    nnz = n * d // 2
    perm = torch.randperm(n * d)[:nnz]
    rows, cols = perm // d, perm % d
    idx = torch.argsort(rows, stable=True)
    mask = kt.SparseMask(indices=torch.stack([rows[idx], cols[idx]]), values=torch.ones(nnz), dense_shape=(n, d),
                         sparsity_ratio=1.0 - nnz / (n * d))
    _gather_case(se, "ref_gather", weight, mask,
                 [torch.tensor([0, 3, 5, 7, 9]), torch.tensor([2, 2, 5, 5, 2]), torch.tensor([], dtype=torch.int64)])
    empty = kt.SparseMask(indices=torch.zeros(2, 0, dtype=torch.int64), values=torch.zeros(0), dense_shape=(10, 8),
                          sparsity_ratio=1.0)
    _gather_case(se, "ref_gather_empty_mask", weight, empty, [torch.tensor([0, 1])])

    # -- an unsorted mask with rows of every length, repeated ids
    g = torch.Generator().manual_seed(7)
    n, d = 300, 48
    dens = torch.rand(n, generator=g)  # per-row density, some rows empty or full
    dens[:5] = 0.0
    dens[5:10] = 1.0
    keep = torch.rand(n, d, generator=g) < dens[:, None]
    r, c = keep.nonzero(as_tuple=True)
    sh = torch.randperm(r.numel(), generator=g)
    mask = kt.SparseMask(indices=torch.stack([r[sh], c[sh]]), values=torch.ones(r.numel()), dense_shape=(n, d),
                         sparsity_ratio=1.0 - r.numel() / (n * d))
    weight = torch.randn(n, d, generator=g)
    _gather_case(se, "unsorted_gather", weight, mask,
                 [torch.randint(0, n, (200,), generator=g), torch.arange(n)])

    # -- scatter: the reference's unit tests (test_sparse_embedding_ops.py:161-215)
    torch.manual_seed(42)
    grad = torch.randn(4, 8)
    _scatter_case(se, "ref_scatter", grad, torch.tensor([1, 3, 5]), torch.tensor([1, 3, 1, 5]), 10, 8)
    _scatter_case(se, "ref_scatter_inactive", torch.ones(2, 4), torch.tensor([0]), torch.tensor([0, 2]), 6, 4)

    # -- scatter: skewed batch (hot rows repeated many times), part of the
    #    batch inactive, active rows absent from the batch
    g = torch.Generator().manual_seed(11)
    n, d, b = 500, 40, 1000
    ranks = torch.arange(1, n + 1, dtype=torch.float64)
    p = (1.0 / ranks) / (1.0 / ranks).sum()
    batch = torch.multinomial(p, b, replacement=True, generator=g)
    uniq = torch.unique(batch)
    active = torch.unique(torch.cat([uniq[torch.rand(uniq.numel(), generator=g) < 0.7],
                                     torch.randint(0, n, (20,), generator=g)]))
    _scatter_case(se, "skewed_scatter", torch.randn(b, d, generator=g), active, batch, n, d)
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
