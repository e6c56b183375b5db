"""Full-size parity: every named workload at the size the benchmark times.

For each workload the problem is generated exactly as ``bench.py`` generates
it (same seed, on the device), the BSR matrix is built on the device and
checked bit for bit against the oracle's stable row sort and row offsets,
and the SpMM runs with the launch configuration the benchmark uses.  Then
the WHOLE result is compared with the oracle (the reference's arithmetic,
kairo/ops/spmm.py:108-134, on fp32-widened inputs):

- the relative Frobenius error of the whole matrix is within TOL, and
- so is the relative error of every single block-row, so that one wrong
  block-row (a split row summed wrongly, an unwritten row) cannot hide in
  the norm of a 262144-row matrix.

Covering every block-row covers every row the row-split schedule cuts over
CTAs, including the 4096-block rows of the Zipf workload and the first and
last rows of every chunk group.  The device error word must stay clean.
"""

from __future__ import annotations

import pytest
import torch

from oracle import oracle
from kairo_b200 import _lib
from kairo_b200.ops import block_sparse_mm_bsr, bsr_from_tiles, describe, sparse_linear
from kairo_b200.workloads import WORKLOADS, block_row_errors, generate, rel_fro_chunked

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

TOL = 1e-3  # relative Frobenius error bar, whole matrix and per block-row
DEV = "cuda"


def _host_bsr_check(p, a):
    """The device BSR build equals the oracle's stable sort + row offsets."""
    s = p.spec
    perm, rows_s, cols_s = oracle.sort_coo_by_row(p.mask.indices[0], p.mask.indices[1], s.nbr)
    assert torch.equal(a.row_ptr.cpu().to(torch.int64), oracle.row_offsets(rows_s, s.nbr))
    assert torch.equal(a.col_idx.cpu().to(torch.int64), cols_s)
    got = torch.arange(p.mask.nnz) if a.blk_idx is None else a.blk_idx.cpu().to(torch.int64)
    assert torch.equal(got, perm)


def _oracle_rows(a, b_host, m, k, n):
    """C = A @ B over every block-row, by the oracle, from host copies."""
    return oracle.spmm_bsr_rows(a.row_ptr.cpu(), a.col_idx.cpu(), None if a.blk_idx is None else a.blk_idx.cpu(),
                                a.blocks.cpu(), b_host, m, k, n, list(range(a.nbr)))[:m]


def _workspace_clean():
    ws = _lib.workspace(0, torch.device(DEV))
    assert _lib.read_workspace_error(ws) == 0


def _assert_close(c, ref, bm, what):
    err = rel_fro_chunked(c, ref)
    rows = block_row_errors(c, ref, bm)
    worst = int(torch.argmax(rows))
    assert err <= TOL, f"{what}: relative error {err:.3e}"
    assert float(rows[worst]) <= TOL, f"{what}: block-row {worst} relative error {float(rows[worst]):.3e}"


@pytest.mark.parametrize("name", ["fp32_uniform", "fp16_uniform", "fp16_zipf", "bf16_uniform"])
def test_standard_workload_full_size(name):
    spec = WORKLOADS[name]
    p = generate(spec, seed=0, device=DEV)
    a = bsr_from_tiles(p.tiles, p.row_ids, p.col_ids, (spec.m, spec.k))
    _host_bsr_check(p, a)
    plan = describe(a, spec.n)
    c = block_sparse_mm_bsr(a, p.b)
    torch.cuda.synchronize()
    _workspace_clean()
    ref = _oracle_rows(a, p.b.cpu(), spec.m, spec.k, spec.n)
    _assert_close(c.cpu(), ref, spec.block, f"{name} ({plan['kernel']}, {plan['schedule']}, grid {plan['grid']})")


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_linear_workload_full_size(out_dtype):
    """Y = X W^T with W 8192 x 32768 (64 x 64 blocks, top 20 % by norm) and
    a batch of 8192: the fp32-output mode against the oracle, and the bf16
    output against the oracle rounded to bf16 (the rounding alone is about
    2e-3 relative, above the fp32 bar)."""
    spec = WORKLOADS["bf16_linear"]
    p = generate(spec, seed=0, device=DEV)
    w = bsr_from_tiles(p.tiles, p.row_ids, p.col_ids, (spec.m, spec.k))
    _host_bsr_check(p, w)
    y = sparse_linear(p.b, w, out_dtype=out_dtype)
    torch.cuda.synchronize()
    _workspace_clean()
    # the oracle computes C = W @ X^T (M x N); Y = C^T
    ref = _oracle_rows(w, p.b.cpu().t().contiguous(), spec.m, spec.k, spec.n).t()
    if out_dtype == torch.bfloat16:
        ref = ref.to(torch.bfloat16).float()
    _assert_close(y.float().cpu().t().contiguous(), ref.t().contiguous(), spec.block, f"bf16_linear -> {out_dtype}")


@pytest.mark.parametrize("name", ["fp16_zipf", "bf16_uniform"])
def test_unsorted_build_full_size(name):
    """The reference's stable row sort on the device for a shuffled tile
    list of the full-size masks: 4096-block rows (shared-memory bucket sort)
    and 335544 tiles in ~41-block rows (warp sort)."""
    spec = WORKLOADS[name]
    p = generate(spec, seed=0, device=DEV)
    g = torch.Generator(device=DEV).manual_seed(11)
    perm = torch.randperm(p.mask.nnz, generator=g, device=DEV)
    rows, cols = p.row_ids[perm].contiguous(), p.col_ids[perm].contiguous()
    tiles = p.tiles[perm].contiguous()
    a = bsr_from_tiles(tiles, rows, cols, (spec.m, spec.k))
    ref_perm, rows_s, cols_s = oracle.sort_coo_by_row(rows.cpu(), cols.cpu(), spec.nbr)
    assert torch.equal(a.row_ptr.cpu().to(torch.int64), oracle.row_offsets(rows_s, spec.nbr))
    assert torch.equal(a.col_idx.cpu().to(torch.int64), cols_s)
    assert torch.equal(a.blk_idx.cpu().to(torch.int64), ref_perm)
    # The product through the permutation (blocks gathered by blk_idx; the
    # stable sort keeps the shuffled order inside a row, so the sums run in
    # another order than for the sorted list) against the oracle on the
    # shuffled list's own BSR order.
    c = block_sparse_mm_bsr(a, p.b)
    torch.cuda.synchronize()
    _workspace_clean()
    ref = _oracle_rows(a, p.b.cpu(), spec.m, spec.k, spec.n)
    _assert_close(c.cpu(), ref, spec.block, f"{name}, shuffled tile list")
