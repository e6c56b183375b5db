"""Parity of the CUDA path with the CPU oracle (the reference's algorithm).

Indexing and construction (BSR row_ptr / col_idx / block order, dense->tile
gather) must be bit-exact.  Numerical output must be within a relative
Frobenius error of 1e-3 of the fp32-accumulated oracle (TOL below).
"""

from __future__ import annotations

import pytest
import torch

from oracle import oracle
from kairo_b200 import _C, _lib
from kairo_b200.ops import KernelConfig, block_sparse_mm, block_sparse_mm_bsr, bsr_from_tiles, sparse_linear
from kairo_b200.ops.spmm import _dense_to_block_sparse
from kairo_b200.types import SparseMask
from kairo_b200.workloads import WORKLOADS, WorkloadSpec, generate
from tests.conftest import rel_fro

pytestmark = pytest.mark.gpu

TOL = 1e-3  # relative Frobenius error bar of the SpMM output vs the fp32 oracle
DEV = "cuda"


def _to_dev(p):
    return p.tiles.to(DEV), p.row_ids.to(DEV), p.col_ids.to(DEV), p.b.to(DEV)


def _oracle_c(p):
    s = p.spec
    return oracle.spmm_tiles(p.tiles, p.row_ids, p.col_ids, p.b, s.m, s.k, s.n, s.block)


def _shuffle(p, seed=7):
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(p.mask.nnz, generator=g)
    mask = SparseMask(indices=p.mask.indices[:, perm], values=p.mask.values[perm], dense_shape=p.mask.dense_shape,
                      sparsity_ratio=p.mask.sparsity_ratio)
    return type(p)(spec=p.spec, mask=mask, tiles=p.tiles[perm].contiguous(), b=p.b)


# --------------------------------------------------------------- construction

@pytest.mark.parametrize("shuffled", [False, True])
@pytest.mark.parametrize("shape", [(64, 64, 16, 0.5), (1024, 2048, 16, 0.9), (4096, 4096, 32, 0.97)])
def test_bsr_build_bit_exact(shape, shuffled):
    m, k, bs, sp = shape
    p = generate(WorkloadSpec("t", torch.float16, m, k, 32, bs, sp), seed=3)
    if shuffled:
        p = _shuffle(p)
    tiles, rows, cols, _ = _to_dev(p)
    a = bsr_from_tiles(tiles, rows, cols, (m, k))
    nbr = (m + bs - 1) // bs
    perm, rows_s, cols_s = oracle.sort_coo_by_row(p.mask.indices[0], p.mask.indices[1], nbr)
    offs = oracle.row_offsets(rows_s, nbr)
    assert torch.equal(a.row_ptr.cpu().to(torch.int64), offs)
    assert torch.equal(a.col_idx.cpu().to(torch.int64), cols_s)
    got_perm = torch.arange(p.mask.nnz) if a.blk_idx is None else a.blk_idx.cpu().to(torch.int64)
    assert torch.equal(got_perm, perm)
    assert (a.blk_idx is None) == (not shuffled)


def test_bsr_build_zipf_long_rows_unsorted():
    p = _shuffle(generate(WORKLOADS["fp16_zipf"].scaled(4096, 4096, 32), seed=1))
    tiles, rows, cols, _ = _to_dev(p)
    a = bsr_from_tiles(tiles, rows, cols, (4096, 4096))
    perm, rows_s, cols_s = oracle.sort_coo_by_row(p.mask.indices[0], p.mask.indices[1], 256)
    assert torch.equal(a.row_ptr.cpu().to(torch.int64), oracle.row_offsets(rows_s, 256))
    assert torch.equal(a.col_idx.cpu().to(torch.int64), cols_s)
    assert torch.equal(a.blk_idx.cpu().to(torch.int64), perm)


@pytest.mark.parametrize("nbr,nbc,per_row", [(50000, 64, 3), (40, 8192, 2000), (20000, 256, 40)])
def test_bsr_build_unsorted_many_and_long_rows(nbr, nbc, per_row):
    """Unsorted tile lists: more block-rows than one CTA scans (the
    multi-CTA scan), rows of up to 32 tiles (sorted in registers by a warp)
    and longer rows (sorted in shared memory)."""
    g = torch.Generator().manual_seed(nbr)
    lens = torch.randint(0, 2 * per_row + 1, (nbr,), generator=g).clamp(max=nbc)
    rows = torch.repeat_interleave(torch.arange(nbr), lens)
    cols = torch.cat([torch.randperm(nbc, generator=g)[:int(n)] for n in lens])
    sh = torch.randperm(rows.numel(), generator=g)
    rows, cols = rows[sh].contiguous(), cols[sh].contiguous()
    tiles = torch.zeros(rows.numel(), 16, 16, dtype=torch.float16, device=DEV)
    a = bsr_from_tiles(tiles, rows.to(DEV), cols.to(DEV), (nbr * 16, nbc * 16))
    perm, rows_s, cols_s = oracle.sort_coo_by_row(rows, cols, nbr)
    assert torch.equal(a.row_ptr.cpu().to(torch.int64), oracle.row_offsets(rows_s, nbr))
    assert torch.equal(a.col_idx.cpu().to(torch.int64), cols_s)
    assert torch.equal(a.blk_idx.cpu().to(torch.int64), perm)
    assert a.max_row_blocks == int(lens.max())


def test_bsr_build_rejects_bad_ids():
    tiles = torch.zeros(2, 16, 16, device=DEV, dtype=torch.float16)
    rows = torch.tensor([0, 5], device=DEV, dtype=torch.int32)
    cols = torch.tensor([0, 0], device=DEV, dtype=torch.int32)
    with pytest.raises(_lib.KairoError, match="outside the block grid"):
        bsr_from_tiles(tiles, rows, cols, (32, 32))


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape", [(64, 64, 16), (40, 56, 16), (100, 70, 32)])
def test_dense_to_tiles_bit_exact(dtype, shape):
    m, k, tile = shape
    g = torch.Generator().manual_seed(5)
    A = torch.randn(m, k, generator=g).to(dtype)
    nbr, nbc = (m + tile - 1) // tile, (k + tile - 1) // tile
    perm = torch.randperm(nbr * nbc, generator=g)[: max(1, nbr * nbc // 2)]
    rows, cols = perm // nbc, perm % nbc
    mask = SparseMask(torch.stack([rows, cols]), torch.ones(perm.numel()), (nbr, nbc), 0.5)
    dmask = SparseMask(mask.indices.to(DEV), mask.values.to(DEV), mask.dense_shape, 0.5)
    tiles, r32, c32 = _dense_to_block_sparse(A.to(DEV), dmask, tile)
    ref = oracle.dense_to_tiles(A, rows, cols, tile)
    assert r32.dtype == torch.int32 and c32.dtype == torch.int32
    assert torch.equal(tiles.cpu().view(torch.int16 if dtype != torch.float32 else torch.int32),
                       ref.view(torch.int16 if dtype != torch.float32 else torch.int32))


# --------------------------------------------------------------- SpMM numerics

TC_CASES = [
    # dtype, bs, m, k, n, sparsity, mask, n_tile, num_ctas, row_cost
    (torch.float16, 16, 512, 512, 128, 0.9, "uniform", 0, 0, 0),
    (torch.float16, 32, 1024, 1024, 256, 0.95, "uniform", 128, 0, 0),
    (torch.float16, 32, 1024, 1024, 512, 0.95, "uniform", 256, 0, 0),
    (torch.bfloat16, 32, 2048, 2048, 256, 0.99, "uniform", 0, 0, 0),
    (torch.bfloat16, 64, 512, 1024, 384, 0.8, "uniform", 256, 0, 0),
    (torch.float16, 64, 512, 512, 128, 0.5, "uniform", 128, 7, 1),
    (torch.float16, 16, 2048, 2048, 128, 0.99, "zipf", 0, 0, 0),
    (torch.float16, 16, 2048, 2048, 128, 0.99, "zipf", 0, 5, 2),
    (torch.bfloat16, 32, 1000, 1000, 200, 0.9, "uniform", 0, 0, 0),   # ragged M, K, N
    (torch.float16, 16, 300, 4000, 72, 0.7, "uniform", 0, 3, 3),      # ragged N < 128, long rows
    (torch.bfloat16, 16, 64, 64, 256, 0.0, "uniform", 256, 2, 1),      # fully dense block grid
]


@pytest.mark.parametrize("case", TC_CASES, ids=lambda c: f"{str(c[0])[6:]}-bs{c[1]}-{c[2]}x{c[3]}x{c[4]}-"
                                                      f"s{c[5]}-{c[6]}-nt{c[7]}-g{c[8]}-r{c[9]}")
def test_tcgen05_spmm_vs_oracle(case):
    dtype, bs, m, k, n, sp, mk, n_tile, num_ctas, row_cost = case
    spec = WorkloadSpec("t", dtype, m, k, n, bs, sp, mask=mk)
    p = generate(spec, seed=11)
    tiles, rows, cols, b = _to_dev(p)
    a = bsr_from_tiles(tiles, rows, cols, (m, k))
    cfg = KernelConfig(kernel="tcgen05", n_tile=n_tile, num_ctas=num_ctas, row_cost=row_cost)
    c = block_sparse_mm_bsr(a, b, config=cfg, check=True)
    ref = _oracle_c(p)
    err = rel_fro(c, ref)
    assert err <= TOL, f"relative Frobenius error {err:.3e}"
    # determinism: a second launch gives identical bits
    c2 = block_sparse_mm_bsr(a, b, config=cfg, check=True)
    assert torch.equal(c, c2)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape", [(256, 256, 64, 16), (4096, 4096, 256, 16), (512, 512, 200, 16), (130, 90, 33, 32),
                                   (256, 256, 128, 64)])
def test_simt_spmm_vs_oracle(dtype, shape):
    m, k, n, bs = shape
    spec = WorkloadSpec("t", dtype, m, k, n, bs, 0.9 if m > 1000 else 0.6)
    p = generate(spec, seed=2)
    tiles, rows, cols, b = _to_dev(p)
    a = bsr_from_tiles(tiles, rows, cols, (m, k))
    c = block_sparse_mm_bsr(a, b, config=KernelConfig(kernel="simt"), check=True)
    err = rel_fro(c, _oracle_c(p))
    assert err <= TOL, f"relative Frobenius error {err:.3e}"


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("bm,bk", [(16, 8), (8, 16), (24, 32), (64, 16)])
def test_simt_spmm_rectangular_blocks(dtype, bm, bk):
    """Non-square blocks (bk outside 16/32/64 takes the per-block kernel, the
    others the row-staged one with bm below its register bound), against a
    dense float64 product of the same BSR matrix."""
    g = torch.Generator().manual_seed(bm * 100 + bk)
    nbr, nbc, n = 40, 30, 100
    keep = torch.rand(nbr, nbc, generator=g) < 0.3
    rows, cols = keep.nonzero(as_tuple=True)
    tiles = torch.randn(rows.numel(), bm, bk, generator=g).to(dtype)
    b = torch.randn(nbc * bk, n, generator=g).to(dtype)
    a = bsr_from_tiles(tiles.to(DEV), rows.to(DEV), cols.to(DEV), (nbr * bm, nbc * bk))
    c = block_sparse_mm_bsr(a, b.to(DEV), config=KernelConfig(kernel="simt"), check=True)
    dense = torch.zeros(nbr * bm, nbc * bk, dtype=torch.float64)
    for t in range(rows.numel()):
        r, q = int(rows[t]), int(cols[t])
        dense[r * bm:(r + 1) * bm, q * bk:(q + 1) * bk] = tiles[t].double()
    ref = dense @ b.double()
    assert rel_fro(c, ref) <= TOL


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", [(256, 512, 256, 64, 0.8, 256), (512, 1024, 300, 32, 0.9, 128),
                                   (128, 256, 128, 16, 0.5, 0)])
def test_sparse_linear_vs_oracle(out_dtype, shape):
    m, k, n, bs, sp, n_tile = shape
    spec = WorkloadSpec("t", torch.bfloat16, m, k, n, bs, sp, mask="magnitude",
                                              layout="linear", a_std=0.02)
    p = generate(spec, seed=4)
    tiles, rows, cols, x = _to_dev(p)
    w = bsr_from_tiles(tiles, rows, cols, (m, k))
    y = sparse_linear(x, w, out_dtype=out_dtype, config=KernelConfig(n_tile=n_tile), check=True)
    # Y = X W^T = (W X^T)^T: the oracle computes C = W @ X^T
    ref = oracle.spmm_tiles(p.tiles, p.row_ids, p.col_ids, p.b.t().contiguous(), m, k, n, bs).t()
    if out_dtype == torch.float32:
        assert rel_fro(y, ref) <= TOL
    else:
        # bf16 output: compare with the oracle rounded to bf16 (the rounding
        # alone is ~2e-3 relative, above the fp32 bar)
        assert rel_fro(y.float(), ref.to(torch.bfloat16).float()) <= TOL


def test_acc_spmm_forward_unsorted_fp16():
    spec = WorkloadSpec("t", torch.float16, 512, 768, 96, 32, 0.8)
    p = _shuffle(generate(spec, seed=9))
    tiles, rows, cols, b = _to_dev(p)
    c = _C.acc_spmm_forward(tiles, rows, cols, b, 512, 768, 96, p.mask.nnz, 32, 32)
    assert c.dtype == torch.float32
    assert rel_fro(c, _oracle_c(p)) <= TOL


def test_acc_spmm_forward_fp32_reference_case():
    """The reference's own CUDA test (tests/ops/test_spmm_ops.py:236-258)."""
    torch.manual_seed(42)
    M, K, N, tile = 32, 32, 16, 16
    A = torch.randn(M, K)
    B = torch.randn(K, N)
    g = torch.Generator().manual_seed(42)
    perm = torch.randperm(4, generator=g)[:2]
    rows, cols = perm // 2, perm % 2
    order = torch.argsort(rows, stable=True)
    mask = SparseMask(torch.stack([rows[order], cols[order]]), torch.ones(2), (2, 2), 0.5)
    tiles = oracle.dense_to_tiles(A, mask.indices[0], mask.indices[1], tile)
    cpu = oracle.spmm_tiles(tiles, mask.indices[0], mask.indices[1], B, M, K, N, tile)
    dmask = SparseMask(mask.indices.cuda(), mask.values.cuda(), mask.dense_shape, mask.sparsity_ratio)
    out = block_sparse_mm(A.cuda(), B.cuda(), dmask, tile_size=tile)
    assert out.device.type == "cuda"
    assert torch.allclose(cpu, out.cpu(), atol=1e-3)


@pytest.mark.parametrize("case", [(torch.bfloat16, 32, 1024, 2048, 1024, 0.95, (256, 512)),
                                  (torch.float16, 16, 512, 1024, 384, 0.9, (128, 384)),
                                  (torch.float32, 16, 256, 512, 512, 0.8, (256, 512))])
def test_spmm_on_a_column_slice_of_b(case):
    """A rank of the multi-GPU grid multiplies by a column slice of the full
    B: a strided view (leading dimension N, base offset c0) into a C tile."""
    dtype, bs, m, k, n, sp, (c0, c1) = case
    p = generate(WorkloadSpec("t", dtype, m, k, n, bs, sp), seed=13)
    tiles, rows, cols, b = _to_dev(p)
    a = bsr_from_tiles(tiles, rows, cols, (m, k))
    view = b[:, c0:c1]
    assert view.stride(0) == n and not view.is_contiguous()
    c = block_sparse_mm_bsr(a, view, check=True)
    ref = oracle.spmm_tiles(p.tiles, p.row_ids, p.col_ids, p.b[:, c0:c1].contiguous(), m, k, c1 - c0, bs)
    assert rel_fro(c, ref) <= TOL


def test_block_sparse_mm_out_dtype():
    """out_dtype=None / float32 give the fp32 product; A's dtype rounds it once."""
    M, K, N, tile = 128, 96, 64, 32
    g = torch.Generator().manual_seed(8)
    A = torch.randn(M, K, generator=g).to(torch.bfloat16)
    B = torch.randn(K, N, generator=g).to(torch.bfloat16)
    keep = torch.rand(M // tile, K // tile, generator=g) < 0.6
    r, c = keep.nonzero(as_tuple=True)
    mask = SparseMask(torch.stack([r, c]).cuda(), torch.ones(r.numel()).cuda(), (M // tile, K // tile), 0.4)
    c32 = block_sparse_mm(A.cuda(), B.cuda(), mask, tile_size=tile)
    assert c32.dtype == torch.float32
    assert torch.equal(block_sparse_mm(A.cuda(), B.cuda(), mask, tile_size=tile, out_dtype=torch.float32), c32)
    cb = block_sparse_mm(A.cuda(), B.cuda(), mask, tile_size=tile, out_dtype=torch.bfloat16)
    assert cb.dtype == torch.bfloat16 and torch.equal(cb, c32.to(torch.bfloat16))
    with pytest.raises(TypeError):
        block_sparse_mm(A.cuda(), B.cuda(), mask, tile_size=tile, out_dtype=torch.float16)


def test_empty_and_zero_rows():
    spec = WorkloadSpec("t", torch.float16, 256, 256, 128, 32, 0.97)
    p = generate(spec, seed=1)
    tiles, rows, cols, b = _to_dev(p)
    a = bsr_from_tiles(tiles, rows, cols, (256, 256))
    c = torch.full((256, 128), float("nan"), device=DEV)
    block_sparse_mm_bsr(a, b, out=c, check=True)
    assert torch.isfinite(c).all()
    assert rel_fro(c, _oracle_c(p)) <= TOL
    # empty matrix: all zeros written
    e = bsr_from_tiles(tiles[:0], rows[:0], cols[:0], (256, 256))
    c.fill_(float("nan"))
    block_sparse_mm_bsr(e, b, out=c)
    assert (c == 0).all()


def test_config_sequence_on_one_workspace():
    """Launches with different grid sizes, chunk counts and kernels share one
    workspace; every result must stay correct (split-row counters are never
    overwritten by another launch's partial tiles)."""
    runs = [
        (WorkloadSpec("t", torch.float16, 512, 512, 128, 64, 0.5), KernelConfig(num_ctas=7, row_cost=1)),
        (WorkloadSpec("t", torch.float16, 2048, 2048, 128, 16, 0.99, mask="zipf"), KernelConfig()),
        (WorkloadSpec("t", torch.float16, 512, 768, 128, 32, 0.8), KernelConfig(num_ctas=3)),
        (WorkloadSpec("t", torch.float16, 512, 768, 128, 32, 0.8), KernelConfig(kernel="simt")),
        (WorkloadSpec("t", torch.bfloat16, 1000, 1000, 200, 32, 0.9), KernelConfig()),
        (WorkloadSpec("t", torch.float16, 512, 768, 512, 32, 0.8), KernelConfig(n_tile=128, num_ctas=16)),
        (WorkloadSpec("t", torch.float16, 512, 768, 128, 32, 0.8), KernelConfig()),
    ]
    for spec, cfg in runs * 2:
        p = generate(spec, seed=21)
        tiles, rows, cols, b = _to_dev(p)
        a = bsr_from_tiles(tiles, rows, cols, (spec.m, spec.k))
        c = torch.full((spec.m, spec.n), float("nan"), device=DEV)
        block_sparse_mm_bsr(a, b, out=c, config=cfg, check=True)
        assert rel_fro(c, _oracle_c(p)) <= TOL, (spec, cfg)


def test_workspace_error_word_clean():
    spec = WorkloadSpec("t", torch.float16, 512, 512, 256, 32, 0.9)
    p = generate(spec, seed=1)
    tiles, rows, cols, b = _to_dev(p)
    a = bsr_from_tiles(tiles, rows, cols, (512, 512))
    block_sparse_mm_bsr(a, b)
    ws = _lib.workspace(0, torch.device(DEV))
    assert _lib.read_workspace_error(ws, clear=False) == 0


# The opt-in split-bf16 kernel takes fp32 A and B through the tcgen05 kernel
# as hi·hi + hi·lo + lo·hi of a bf16 hi/lo split; its error is about 1e-5
# relative (the dropped lo·lo term), so it is held to a bar ten times tighter
# than the 1e-3 parity bar.
SPLIT_TOL = 1e-4


@pytest.mark.parametrize("shape", [(4096, 4096, 256, 16), (512, 512, 200, 32), (256, 256, 128, 64),
                                   (130, 90, 64, 16)])
def test_split_bf16_spmm_vs_oracle(shape):
    m, k, n, bs = shape
    spec = WorkloadSpec("t", torch.float32, m, k, n, bs, 0.9 if m > 1000 else 0.6)
    p = generate(spec, seed=3)
    tiles, rows, cols, b = _to_dev(p)
    a = bsr_from_tiles(tiles, rows, cols, (m, k))
    cfg = KernelConfig(kernel="split_bf16")
    from kairo_b200.ops import describe
    assert describe(a, n, config=cfg)["kernel"] == "split_bf16"
    c = block_sparse_mm_bsr(a, b, config=cfg, check=True)
    err = rel_fro(c, _oracle_c(p))
    assert err <= SPLIT_TOL, f"relative Frobenius error {err:.3e}"
    assert torch.equal(c, block_sparse_mm_bsr(a, b, config=cfg, check=True))


def test_split_bf16_spmm_unsupported():
    g = torch.Generator().manual_seed(4)
    tiles = torch.randn(3, 16, 8, generator=g)
    a = bsr_from_tiles(tiles.to(DEV), torch.tensor([0, 1, 1]).to(DEV), torch.tensor([0, 0, 1]).to(DEV), (32, 16))
    with pytest.raises(_lib.KairoError):
        block_sparse_mm_bsr(a, torch.randn(16, 64, device=DEV), config=KernelConfig(kernel="split_bf16"))
    sq = bsr_from_tiles(torch.randn(2, 16, 16, generator=g).to(torch.bfloat16).to(DEV),
                        torch.tensor([0, 1]).to(DEV), torch.tensor([0, 0]).to(DEV), (32, 16))
    with pytest.raises(_lib.KairoError):
        block_sparse_mm_bsr(sq, torch.randn(16, 64, device=DEV).to(torch.bfloat16),
                            config=KernelConfig(kernel="split_bf16"))
