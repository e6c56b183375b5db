"""Generates the golden fixtures of the SpMM path from the reference itself.

Usage (needs the reference source tree; run where it is mounted):
    python tests/golden/make_golden.py --ref <path of the reference source tree>

The script imports the reference's own ``kairo`` package (its pure-PyTorch CPU
path) and records, for seeded inputs:
  * _dense_to_block_sparse (kairo/ops/spmm.py:16-55) -> tiles, int32 ids
  * the stable row sort of _sort_coo_by_row (kairo/ops/sparse_embedding.py:
    49-56) -> perm, sorted rows/cols; _coo_to_row_offsets (:23-46) -> offsets
  * _block_sparse_mm_fallback (kairo/ops/spmm.py:108-134) on fp32-upcast
    inputs -> C (fp32)
  * block_sparse_mm (kairo/ops/spmm.py:58-105) on CPU for the fp32 dense cases
Each case is saved as tests/golden/<name>.pt (a dict of CPU tensors and ints).
The inputs of the reference's own unit tests (tests/ops/test_spmm_ops.py) are
regenerated here with the same seeds and draw order.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent


def _ref_modules(ref: Path):
    sys.path.insert(0, str(ref))
    import kairo.ops.sparse_embedding as se  # noqa: E402
    import kairo.ops.spmm as spmm  # noqa: E402
    import kairo.types as ktypes  # noqa: E402

    sys.path.pop(0)
    return spmm, se, ktypes


def _make_block_mask(ktypes, nbr, nbc, sparsity, seed=42, sort=True):
    """Same draws as tests/ops/test_spmm_ops.py:21-44 (sort=True) and
    benchmarks/bench_spmm.py:14-35 (sort=False)."""
    torch.manual_seed(seed)
    total = nbr * nbc
    nnz = max(1, int(total * (1.0 - sparsity)))
    perm = torch.randperm(total)[:nnz]
    rows = perm // nbc
    cols = perm % nbc
    if sort:
        idx = torch.argsort(rows, stable=True)
        rows, cols = rows[idx], cols[idx]
    indices = torch.stack([rows, cols]).to(torch.int64)
    return ktypes.SparseMask(indices=indices, values=torch.ones(nnz), dense_shape=(nbr, nbc),
                             sparsity_ratio=sparsity)


def _record(spmm, se, ktypes, name, *, mask, tile, M, K, N, B, A=None, tiles=None):
    out = {"name": name, "tile": tile, "M": M, "K": K, "N": N, "torch_version": torch.__version__,
           "mask_indices": mask.indices.clone(), "mask_shape": tuple(mask.dense_shape), "B": B.clone()}
    if A is not None:
        out["A"] = A.clone()
        t, r, c = spmm._dense_to_block_sparse(A, mask, tile)
        out["tiles"], out["tile_row_ids"], out["tile_col_ids"] = t.clone(), r.clone(), c.clone()
        if A.dtype == torch.float32:
            out["C_op"] = spmm.block_sparse_mm(A, B, mask, tile_size=tile).clone()
    else:
        out["tiles"] = tiles.clone()
        out["tile_row_ids"] = mask.indices[0].to(torch.int32)
        out["tile_col_ids"] = mask.indices[1].to(torch.int32)
    rows_s, cols_s = se._sort_coo_by_row(mask)
    out["perm"] = torch.argsort(mask.indices[0], stable=True)
    out["rows_sorted"], out["cols_sorted"] = rows_s.clone(), cols_s.clone()
    out["row_offsets"] = se._coo_to_row_offsets(rows_s, mask.dense_shape[0]).clone()
    if out["tiles"].shape[0]:
        out["C_ref"] = spmm._block_sparse_mm_fallback(out["tiles"].float(), out["tile_row_ids"], out["tile_col_ids"],
                                                      B.float(), M, K, N, tile).clone()
    else:
        out["C_ref"] = torch.zeros(M, N)
    torch.save(out, HERE / f"{name}.pt")
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of the reference source tree (read-only)")
    args = ap.parse_args()
    spmm, se, ktypes = _ref_modules(Path(args.ref))
    sys.path.insert(0, str(REPO))
    from kairo_b200.workloads import WORKLOADS, generate  # noqa: E402

    # -- the reference's unit-test inputs (tests/ops/test_spmm_ops.py)
    torch.manual_seed(42)
    A = torch.randn(32, 32)
    mask = _make_block_mask(ktypes, 2, 2, 0.5)
    _record(spmm, se, ktypes, "ref_roundtrip", mask=mask, tile=16, M=32, K=32, N=16, A=A,
            B=torch.zeros(32, 16))

    for sp, name in ((0.0, "ref_dense_mask"), (0.75, "ref_sparse75")):
        torch.manual_seed(42)
        A = torch.randn(32, 32)
        B = torch.randn(32, 16)
        mask = _make_block_mask(ktypes, 2, 2, sp)
        _record(spmm, se, ktypes, name, mask=mask, tile=16, M=32, K=32, N=16, A=A, B=B)

    torch.manual_seed(42)
    A = torch.randn(64, 64)
    B = torch.randn(64, 32)
    mask = _make_block_mask(ktypes, 4, 4, 0.95)
    _record(spmm, se, ktypes, "ref_sparse95", mask=mask, tile=16, M=64, K=64, N=32, A=A, B=B)

    torch.manual_seed(42)
    for tile in (16, 32):
        A = torch.randn(64, 64)
        B = torch.randn(64, 32)
        mask = _make_block_mask(ktypes, 64 // tile, 64 // tile, 0.5)
        _record(spmm, se, ktypes, f"ref_tile{tile}", mask=mask, tile=tile, M=64, K=64, N=32, A=A, B=B)

    mask = ktypes.SparseMask(indices=torch.tensor([[0], [0]], dtype=torch.int64), values=torch.ones(1),
                             dense_shape=(1, 1), sparsity_ratio=0.0)
    _record(spmm, se, ktypes, "ref_eye", mask=mask, tile=16, M=16, K=16, N=16, A=torch.eye(16),
            B=torch.arange(256, dtype=torch.float32).view(16, 16) / 7.0)

    torch.manual_seed(42)
    A = torch.randn(32, 32)
    B = torch.randn(32, 16)
    mask = ktypes.SparseMask(indices=torch.zeros(2, 0, dtype=torch.int64), values=torch.zeros(0),
                             dense_shape=(2, 2), sparsity_ratio=1.0)
    _record(spmm, se, ktypes, "ref_empty", mask=mask, tile=16, M=32, K=32, N=16, A=A, B=B)

    # -- the reference benchmark's unsorted mask (benchmarks/bench_spmm.py:14-35)
    A = torch.randn(256, 256)
    B = torch.randn(256, 48)
    mask = _make_block_mask(ktypes, 16, 16, 0.8, sort=False)
    _record(spmm, se, ktypes, "bench_unsorted", mask=mask, tile=16, M=256, K=256, N=48, A=A, B=B)

    # -- ragged edges: M, K not multiples of the tile
    torch.manual_seed(3)
    A = torch.randn(40, 56)
    B = torch.randn(56, 24)
    mask = _make_block_mask(ktypes, 3, 4, 0.4, seed=3)
    _record(spmm, se, ktypes, "ragged_edges", mask=mask, tile=16, M=40, K=56, N=24, A=A, B=B)
    torch.manual_seed(4)
    A = torch.randn(100, 70).half()
    B = torch.randn(70, 40).half()
    mask = _make_block_mask(ktypes, 4, 3, 0.3, seed=4, sort=False)
    _record(spmm, se, ktypes, "ragged_fp16_unsorted", mask=mask, tile=32, M=100, K=70, N=40, A=A, B=B)

    # -- scaled-down versions of the five workload families (tiles generated
    #    block-wise, as for the full-size sparse matrices)
    for fam, (m, k, n) in {"fp32_uniform": (256, 256, 32), "fp16_uniform": (512, 512, 32),
                           "bf16_linear": (256, 512, 32), "fp16_zipf": (1024, 1024, 32),
                           "bf16_uniform": (2048, 2048, 32)}.items():
        spec = WORKLOADS[fam].scaled(m, k, n)
        p = generate(spec, seed=0)
        mask = ktypes.SparseMask(indices=p.mask.indices, values=p.mask.values, dense_shape=p.mask.dense_shape,
                                 sparsity_ratio=p.mask.sparsity_ratio)
        b = p.b.t().contiguous() if spec.layout == "linear" else p.b
        _record(spmm, se, ktypes, f"wl_{fam}", mask=mask, tile=spec.block, M=m, K=k, N=n, B=b, tiles=p.tiles)
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
