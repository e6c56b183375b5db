"""Band schedule of the tcgen05 SpMM against the CPU oracle.

The band schedule visits each block-row's blocks in column order instead of
BSR order, so its sums differ from the row-split schedule's in rounding only;
both must be within the relative Frobenius bar TOL of the fp32 oracle
(kairo/ops/spmm.py:108-134 restated in oracle/).  Cases cover every block
size and sub-tile count, both layouts, ragged shapes, empty rows and items,
unsorted tile input (blk_idx), items longer than the column-sort limit (kept
in BSR order), many item waves (serpentine order) and the schedule choice.
"""

from __future__ import annotations

import pytest
import torch

from oracle import oracle
from kairo_b200 import _lib
from kairo_b200.ops import KernelConfig, block_sparse_mm_bsr, bsr_from_tiles, describe, sparse_linear
from kairo_b200.types import BlockSparseMatrix, SparseMask
from kairo_b200.workloads import WorkloadSpec, generate
from tests.conftest import rel_fro

pytestmark = pytest.mark.gpu

TOL = 1e-3
DEV = "cuda"


def _oracle_c(p):
    s = p.spec
    return oracle.spmm_tiles(p.tiles, p.row_ids, p.col_ids, p.b, s.m, s.k, s.n, s.block)


def _shuffle(p, seed=7):
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(p.mask.nnz, generator=g)
    mask = SparseMask(indices=p.mask.indices[:, perm], values=p.mask.values[perm], dense_shape=p.mask.dense_shape,
                      sparsity_ratio=p.mask.sparsity_ratio)
    return type(p)(spec=p.spec, mask=mask, tiles=p.tiles[perm].contiguous(), b=p.b)


BAND_CASES = [
    # dtype, bs, m, k, n, sparsity, mask, n_tile, num_ctas, band_rows, shuffled
    (torch.float16, 16, 512, 512, 128, 0.9, "uniform", 0, 0, 0, False),
    (torch.float16, 32, 1024, 1024, 256, 0.95, "uniform", 128, 5, 3, False),    # many waves, double slot
    (torch.float16, 32, 1024, 1024, 512, 0.95, "uniform", 256, 0, 8, False),    # single accumulator set
    (torch.bfloat16, 32, 2048, 2048, 256, 0.99, "uniform", 0, 0, 0, False),
    (torch.bfloat16, 64, 512, 1024, 384, 0.8, "uniform", 256, 0, 4, False),
    (torch.float16, 64, 512, 512, 128, 0.5, "uniform", 128, 7, 2, False),
    (torch.float16, 16, 2048, 2048, 128, 0.99, "zipf", 0, 0, 0, False),
    (torch.bfloat16, 32, 1000, 1000, 200, 0.9, "uniform", 0, 0, 0, False),      # ragged M, K, N
    (torch.float16, 16, 300, 4000, 72, 0.7, "uniform", 0, 3, 5, False),         # N < 128, ragged groups
    (torch.bfloat16, 16, 64, 64, 256, 0.0, "uniform", 256, 2, 0, False),        # fully dense block grid
    (torch.float16, 32, 512, 768, 128, 0.8, "uniform", 0, 0, 0, True),          # unsorted input: blk_idx
    (torch.float16, 32, 256, 256, 128, 0.97, "uniform", 0, 0, 2, False),        # empty rows and items
    (torch.float16, 16, 64, 16384, 128, 0.4, "uniform", 0, 0, 4, False),        # item > sort limit
]


@pytest.mark.parametrize("case", BAND_CASES, ids=lambda c: f"{str(c[0])[6:]}-bs{c[1]}-{c[2]}x{c[3]}x{c[4]}-"
                                                        f"s{c[5]}-{c[6]}-nt{c[7]}-g{c[8]}-R{c[9]}"
                                                        f"{'-shuf' if c[10] else ''}")
def test_band_spmm_vs_oracle(case):
    dtype, bs, m, k, n, sp, mk, n_tile, num_ctas, band_rows, shuffled = case
    spec = WorkloadSpec("t", dtype, m, k, n, bs, sp, mask=mk)
    p = generate(spec, seed=13)
    if shuffled:
        p = _shuffle(p)
    a = bsr_from_tiles(p.tiles.to(DEV), p.row_ids.to(DEV), p.col_ids.to(DEV), (m, k))
    if shuffled:
        assert a.blk_idx is not None
    cfg = KernelConfig(kernel="tcgen05", schedule="bands", n_tile=n_tile, num_ctas=num_ctas, band_rows=band_rows)
    plan = describe(a, n, config=cfg)
    assert plan["schedule"] == "bands" and plan["launches"] == 2
    b = p.b.to(DEV)
    c = torch.full((m, n), float("nan"), device=DEV)
    block_sparse_mm_bsr(a, b, out=c, config=cfg, check=True)
    err = rel_fro(c, _oracle_c(p))
    assert err <= TOL, f"relative Frobenius error {err:.3e}"
    c2 = block_sparse_mm_bsr(a, b, config=cfg, check=True)
    assert torch.equal(c, c2)


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_band_sparse_linear_vs_oracle(out_dtype):
    m, k, n, bs = 256, 512, 256, 64
    spec = WorkloadSpec("t", torch.bfloat16, m, k, n, bs, 0.8, mask="magnitude", layout="linear", a_std=0.02)
    p = generate(spec, seed=4)
    w = bsr_from_tiles(p.tiles.to(DEV), p.row_ids.to(DEV), p.col_ids.to(DEV), (m, k))
    cfg = KernelConfig(schedule="bands", band_rows=2)
    assert describe(w, n, linear=True, config=cfg)["schedule"] == "bands"
    y = sparse_linear(p.b.to(DEV), w, out_dtype=out_dtype, config=cfg, check=True)
    ref = oracle.spmm_tiles(p.tiles, p.row_ids, p.col_ids, p.b.t().contiguous(), m, k, n, bs).t()
    if out_dtype == torch.float32:
        assert rel_fro(y, ref) <= TOL
    else:
        assert rel_fro(y.float(), ref.to(torch.bfloat16).float()) <= TOL


def test_band_and_row_schedules_share_a_workspace():
    """Alternating schedules on one cached workspace stay correct (the band
    kernel's column-order array sits after the row-split counter banks)."""
    spec = WorkloadSpec("t", torch.float16, 1024, 1024, 256, 32, 0.9)
    p = generate(spec, seed=5)
    a = bsr_from_tiles(p.tiles.to(DEV), p.row_ids.to(DEV), p.col_ids.to(DEV), (1024, 1024))
    b = p.b.to(DEV)
    ref = _oracle_c(p)
    for cfg in [KernelConfig(schedule="bands"), KernelConfig(schedule="rows", num_ctas=9),
                KernelConfig(schedule="bands", band_rows=1, num_ctas=4), KernelConfig(schedule="rows")] * 2:
        c = torch.full((1024, 256), float("nan"), device=DEV)
        block_sparse_mm_bsr(a, b, out=c, config=cfg, check=True)
        assert rel_fro(c, ref) <= TOL, cfg


@pytest.mark.parametrize("schedule", ["rows", "bands"])
def test_out_of_range_block_column_is_reported(schedule):
    """A block-column id past the matrix is recorded in the device error word
    (the kernels load column 0 instead, so nothing is read out of bounds)."""
    spec = WorkloadSpec("t", torch.float16, 256, 256, 128, 32, 0.5)
    p = generate(spec, seed=2)
    a = bsr_from_tiles(p.tiles.to(DEV), p.row_ids.to(DEV), p.col_ids.to(DEV), (256, 256))
    bad_cols = a.col_idx.clone()
    bad_cols[3] = a.nbc + 5
    bad = BlockSparseMatrix(row_ptr=a.row_ptr, col_idx=bad_cols, blocks=a.blocks, shape=a.shape,
                            block_size=a.block_size, blk_idx=a.blk_idx)
    with pytest.raises(_lib.KairoDeviceError):
        block_sparse_mm_bsr(bad, p.b.to(DEV), config=KernelConfig(schedule=schedule), check=True)
    # the error is reported once; the next launch on the same workspace is clean
    c = block_sparse_mm_bsr(a, p.b.to(DEV), config=KernelConfig(schedule=schedule), check=True)
    assert rel_fro(c, _oracle_c(p)) <= TOL


def _uniform_rows_matrix(nbr, nbc, per_row, bs, max_row_blocks):
    """Metadata-only BSR (one stored block, every position maps to it) for
    plan queries; no SpMM is run on it."""
    cols = (torch.arange(nbr * per_row, device=DEV, dtype=torch.int32) * 7919) % nbc
    rp = torch.arange(0, nbr * per_row + 1, per_row, device=DEV, dtype=torch.int32)
    blocks = torch.zeros(1, bs, bs, dtype=torch.bfloat16, device=DEV)
    blk = torch.zeros(nbr * per_row, dtype=torch.int32, device=DEV)
    return BlockSparseMatrix(row_ptr=rp, col_idx=cols, blocks=blocks, shape=(nbr * bs, nbc * bs),
                             block_size=(bs, bs), blk_idx=blk, max_row_blocks=max_row_blocks)


def test_schedule_choice():
    """AUTO picks the band schedule when a chunk has fewer block-rows than
    twice the SMs (the row-split schedule would cut most rows) or the block
    grid is at least 10 % dense, with enough items and a row-length hint
    showing similar rows; otherwise rows."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    # many short rows (the 262144^2 case): rows
    a = _uniform_rows_matrix(1024, 8192, 41, 32, max_row_blocks=41)
    assert describe(a, 1024)["schedule"] == "rows"
    assert describe(a, 1024, config=KernelConfig(schedule="bands"))["schedule"] == "bands"
    plan = describe(a, 1024)
    # 32x32 blocks: two CTAs per SM, each with three stages of two 18 KB slots
    assert plan["grid"] == 2 * sms and (plan["stages"], plan["group_blocks"]) == (3, 2)
    # one CTA per SM with the B slice above half of L2: four stages of three slots
    one = describe(a, 1024, config=KernelConfig(ctas_per_sm=1))
    assert one["grid"] == sms and (one["stages"], one["group_blocks"]) == (4, 3)
    # few long rows, many chunks (the linear layer): bands
    few = max(1, sms // 2)
    b = _uniform_rows_matrix(few, 512, 100, 64, max_row_blocks=100)
    assert describe(b, 8192)["schedule"] == "bands"
    # two CTAs per SM by default, each with one 64-row block-row per item
    assert describe(b, 8192)["grid"] == 2 * sms
    assert describe(b, 8192, config=KernelConfig(ctas_per_sm=1))["grid"] == sms
    # ... and one when the caller's band_rows need the whole TMEM
    wide = describe(b, 8192, config=KernelConfig(band_rows=4))
    assert wide["grid"] == sms and wide["rows"] == 4
    # ... but not without the row-length hint, nor with a very long row
    assert describe(_uniform_rows_matrix(few, 512, 100, 64, max_row_blocks=0), 8192)["schedule"] == "rows"
    assert describe(_uniform_rows_matrix(few, 512, 100, 64, max_row_blocks=400), 8192)["schedule"] == "rows"
    a2 = _uniform_rows_matrix(1024, 512, 41, 32, max_row_blocks=41)
    plan2 = describe(a2, 1024, config=KernelConfig(ctas_per_sm=1))
    assert plan2["schedule"] == "rows" and (plan2["stages"], plan2["group_blocks"]) == (3, 4)
    assert (describe(a2, 1024)["stages"], describe(a2, 1024)["group_blocks"]) == (3, 2)
    # many rows on a dense block grid (the transposed linear-layer weight,
    # 20 % of 512 x 128 blocks): bands
    c = _uniform_rows_matrix(512, 128, 26, 64, max_row_blocks=26)
    assert describe(c, 8192)["schedule"] == "bands"


def test_build_reports_longest_row():
    spec = WorkloadSpec("t", torch.float16, 2048, 2048, 128, 16, 0.99, mask="zipf")
    p = generate(spec, seed=3)
    a = bsr_from_tiles(p.tiles.to(DEV), p.row_ids.to(DEV), p.col_ids.to(DEV), (2048, 2048))
    counts = torch.bincount(p.row_ids.long(), minlength=a.nbr)
    assert a.max_row_blocks == int(counts.max())


@pytest.mark.parametrize("per_sm", [1, 2])
@pytest.mark.parametrize("shape", [(512, 2048, 1024, 64, 0.8), (1024, 1024, 512, 32, 0.7)])
def test_band_ctas_per_sm_vs_oracle(shape, per_sm):
    """The band schedule with one and with two resident CTAs per SM (two
    split the TMEM and shared memory: one block-row per item for 64x64
    blocks)."""
    m, k, n, bs, sp = shape
    spec = WorkloadSpec("t", torch.bfloat16, m, k, n, bs, sp)
    p = generate(spec, seed=12)
    a = bsr_from_tiles(p.tiles.to(DEV), p.row_ids.to(DEV), p.col_ids.to(DEV), (m, k))
    cfg = KernelConfig(schedule="bands", ctas_per_sm=per_sm)
    plan = describe(a, n, config=cfg)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    assert plan["schedule"] == "bands" and plan["grid"] <= per_sm * sms
    c = block_sparse_mm_bsr(a, p.b.to(DEV), config=cfg, check=True)
    ref = oracle.spmm_tiles(p.tiles, p.row_ids, p.col_ids, p.b, m, k, n, bs)
    assert rel_fro(c, ref) <= TOL
