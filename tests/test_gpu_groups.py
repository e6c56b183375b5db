"""Row groups (kairo_bsr_stack_build + kairo_bsr_spmm_stacked) on the GPU.

The group tables must equal a host restatement of their definition exactly
(block-rows ordered by block count, longest first, ties by index; each
group's distinct column-blocks ascending, with the mask of the group rows
that have a block there and each block's stored index).  The SpMM must agree
with the fp32 oracle within the relative Frobenius bar of the other parity
tests (TOL), on skewed and uniform masks, both dtypes, every instantiated
(block, n_tile, group size), ragged shapes, rows cut over many CTAs and
empty groups.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle
from kairo_b200 import _lib
from kairo_b200.ops import KernelConfig, block_sparse_mm_bsr, bsr_from_tiles, bsr_row_groups, describe
from kairo_b200.ops import spmm as spmm_mod
from kairo_b200.ops.spmm import _bsr_desc
from kairo_b200.workloads import WORKLOADS, WorkloadSpec, generate
from tests.conftest import rel_fro

pytestmark = pytest.mark.gpu

TOL = 1e-3  # relative Frobenius error bar of the SpMM output vs the fp32 oracle
DEV = "cuda"


def _problem(m, k, n, bs, sp, mask="zipf", dtype=torch.float16, seed=0):
    spec = WorkloadSpec("groups", dtype, m, k, n, bs, sp, mask=mask)
    p = generate(spec, seed=seed)
    a = bsr_from_tiles(p.tiles.to(DEV), p.row_ids.to(DEV), p.col_ids.to(DEV), (m, k))
    return spec, p, a


def _oracle(spec, p):
    return oracle.spmm_tiles(p.tiles, p.row_ids, p.col_ids, p.b, spec.m, spec.k, spec.n, spec.block)


def _host_groups(a, rg):
    """The group tables by their definition, on the host."""
    row_ptr = a.row_ptr.cpu().numpy().astype(np.int64)
    col = a.col_idx.cpu().numpy().astype(np.int64)
    blk = np.arange(a.nnzb) if a.blk_idx is None else a.blk_idx.cpu().numpy().astype(np.int64)
    lens = np.diff(row_ptr)
    order = sorted(range(a.nbr), key=lambda i: (-lens[i], i))
    ngroups = (a.nbr + rg - 1) // rg
    row_map = np.full(ngroups * rg, -1, dtype=np.int64)
    row_map[: a.nbr] = order
    group_ptr, scol, smask, sblk = [0], [], [], []
    for g in range(ngroups):
        cols = {}
        for r in range(rg):
            row = row_map[g * rg + r]
            if row < 0:
                continue
            for p in range(row_ptr[row], row_ptr[row + 1]):
                cols.setdefault(int(col[p]), {})[r] = int(blk[p])
        for c in sorted(cols):
            scol.append(c)
            smask.append(sum(1 << r for r in cols[c]))
            sblk.append(cols[c])
        group_ptr.append(len(scol))
    return row_map, np.array(group_ptr), np.array(scol), np.array(smask), sblk


@pytest.mark.parametrize("rg", [2, 4, 8])
@pytest.mark.parametrize("case", ["zipf", "uniform_shuffled", "empty_rows"])
def test_group_tables_exact(case, rg):
    if case == "zipf":
        _, _, a = _problem(2048, 2048, 128, 16, 0.97)
    elif case == "uniform_shuffled":
        spec = WorkloadSpec("g", torch.float16, 1024, 2048, 128, 32, 0.9)
        p = generate(spec, seed=4)
        g = torch.Generator().manual_seed(5)
        perm = torch.randperm(p.mask.nnz, generator=g)
        a = bsr_from_tiles(p.tiles[perm].to(DEV), p.row_ids[perm].to(DEV), p.col_ids[perm].to(DEV), (1024, 2048))
        assert a.blk_idx is not None
    else:
        # a few non-empty rows among many empty ones, and a ragged group count
        _, _, a = _problem(16 * 37, 1024, 128, 16, 0.995)
    groups = bsr_row_groups(a, rg)
    t = groups.tables()
    row_map, group_ptr, scol, smask, sblk = _host_groups(a, rg)
    assert groups.ngroups == len(group_ptr) - 1
    assert groups.nsuper == len(scol)
    assert np.array_equal(t["row_map"].cpu().numpy(), row_map)
    assert np.array_equal(t["group_ptr"].cpu().numpy(), group_ptr)
    assert np.array_equal(t["super_col"].cpu().numpy(), scol)
    assert np.array_equal(t["super_mask"].cpu().numpy(), smask)
    got_blk = t["super_blk"].cpu().numpy().reshape(-1, rg)
    for q, present in enumerate(sblk):
        for r, b in present.items():
            assert got_blk[q, r] == b


# (block, n, group rows): every instantiated kernel, N of one and two
# 128-column sub-tiles, and a ragged N
_CASES = [(16, 128, 2), (16, 128, 4), (16, 128, 8), (16, 256, 2), (16, 256, 4), (16, 200, 4),
          (32, 128, 2), (32, 128, 4), (32, 256, 2), (32, 96, 4)]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("bs,n,rg", _CASES)
def test_groups_spmm_zipf_vs_oracle(bs, n, rg, dtype):
    spec, p, a = _problem(4096, 4096, n, bs, 0.97 if bs == 16 else 0.95, dtype=dtype)
    cfg = KernelConfig(schedule="groups", group_rows=rg)
    plan = describe(a, n, config=cfg)
    assert plan["schedule"] == "groups" and plan["rows"] == rg
    c = block_sparse_mm_bsr(a, p.b.to(DEV), config=cfg, check=True)
    err = rel_fro(c.cpu(), _oracle(spec, p))
    assert err <= TOL, f"bs={bs} n={n} rg={rg} {dtype}: {err:.3e}"


@pytest.mark.parametrize("num_ctas", [1, 3, 17, 148, 296])
def test_groups_rows_cut_over_ctas(num_ctas):
    """Long groups cut into many pieces (partial tiles summed by the last CTA)."""
    spec, p, a = _problem(2048, 4096, 128, 16, 0.96)
    cfg = KernelConfig(schedule="groups", group_rows=4, num_ctas=num_ctas)
    c = block_sparse_mm_bsr(a, p.b.to(DEV), config=cfg, check=True)
    assert rel_fro(c.cpu(), _oracle(spec, p)) <= TOL


@pytest.mark.parametrize("mask", ["uniform", "zipf"])
def test_groups_ragged_shapes(mask):
    """M, K and N not multiples of the block or the 128-column tile (N a
    multiple of 8: B rows are copied with TMA)."""
    spec, p, a = _problem(1000, 1500, 136, 16, 0.9, mask=mask, dtype=torch.bfloat16)
    c = block_sparse_mm_bsr(a, p.b.to(DEV), config=KernelConfig(schedule="groups", group_rows=4), check=True)
    assert rel_fro(c.cpu(), _oracle(spec, p)) <= TOL


def test_groups_deterministic_and_matches_rows():
    spec, p, a = _problem(4096, 4096, 128, 16, 0.98)
    b = p.b.to(DEV)
    cfg = KernelConfig(schedule="groups", group_rows=4)
    c1 = block_sparse_mm_bsr(a, b, config=cfg, check=True)
    c2 = block_sparse_mm_bsr(a, b, config=cfg, check=True)
    assert torch.equal(c1, c2)
    rows = block_sparse_mm_bsr(a, b, config=KernelConfig(schedule="rows"), check=True)
    assert rel_fro(c1.cpu(), rows.cpu()) <= 1e-5


def test_groups_auto_choice(monkeypatch):
    """AUTO leaves row groups off by default; with the switch on, it takes
    them for a skewed mask and not for a uniform one."""
    spec, p, a = _problem(8192, 8192, 128, 16, 0.99)
    assert describe(a, spec.n)["schedule"] != "groups"
    monkeypatch.setattr(spmm_mod, "_GROUPS_AUTO", True)
    assert describe(a, spec.n)["schedule"] == "groups"
    c = block_sparse_mm_bsr(a, p.b.to(DEV), check=True)
    assert rel_fro(c.cpu(), _oracle(spec, p)) <= TOL
    _, _, u = _problem(8192, 8192, 128, 16, 0.99, mask="uniform")
    assert describe(u, 128)["schedule"] != "groups"


def test_groups_duplicate_columns_rejected():
    """A block-row with two blocks in one column (the reference adds both)
    cannot be stacked: the row-group schedule raises; the default path adds
    both as the reference does."""
    rows = torch.tensor([0, 0, 0, 1, 1] * 40, dtype=torch.int32)
    cols = torch.tensor([3, 3, 5, 1, 2] * 40, dtype=torch.int32)
    tiles = torch.randn(rows.numel(), 16, 16).half()
    m = k = 16 * 8
    a = bsr_from_tiles(tiles.to(DEV), rows.to(DEV), cols.to(DEV), (m, k))
    b = torch.randn(k, 128).half()
    with pytest.raises(_lib.KairoError):
        block_sparse_mm_bsr(a, b.to(DEV), config=KernelConfig(schedule="groups", group_rows=2))
    c = block_sparse_mm_bsr(a, b.to(DEV), check=True)
    ref = oracle.spmm_tiles(tiles, rows, cols, b, m, k, 128, 16)
    assert rel_fro(c.cpu(), ref) <= TOL


def test_groups_empty_and_zero_rows():
    """All-empty groups write zeros over whatever C held."""
    spec, p, a = _problem(16 * 64, 1024, 128, 16, 0.999)
    out = torch.full((spec.m, spec.n), float("nan"), device=DEV)
    c = block_sparse_mm_bsr(a, p.b.to(DEV), out=out, config=KernelConfig(schedule="groups", group_rows=8),
                            check=True)
    assert not torch.isnan(c).any()
    assert rel_fro(c.cpu(), _oracle(spec, p)) <= TOL


def test_groups_bad_block_index_recorded():
    """An out-of-range stored-block index in the group tables is caught by
    the kernel's bounds check (it loads block 0 instead) and reported."""
    spec, p, a = _problem(2048, 2048, 128, 16, 0.97)
    groups = bsr_row_groups(a, 4)
    t = groups.tables()
    mask0 = int(t["super_mask"][0].item())
    r0 = (mask0 & -mask0).bit_length() - 1
    t["super_blk"][r0] = a.blocks.shape[0] + 5
    with pytest.raises(_lib.KairoDeviceError) as ei:
        block_sparse_mm_bsr(a, p.b.to(DEV), config=KernelConfig(schedule="groups", group_rows=4), check=True)
    assert ei.value.code & 0xFF == _lib.DEVERR_BAD_INDEX


def test_groups_c_abi_direct():
    """kairo_bsr_stack_build + kairo_bsr_spmm_stacked through ctypes."""
    spec, p, a = _problem(2048, 2048, 256, 32, 0.95, dtype=torch.bfloat16)
    lib = _lib.lib()
    desc = _bsr_desc(a)
    nbytes = ctypes.c_size_t(0)
    assert lib.kairo_bsr_stack_size(ctypes.byref(desc), 2, ctypes.byref(nbytes)) == 0
    mem = torch.empty(nbytes.value, dtype=torch.uint8, device=DEV)
    st = _lib.KairoBsrStack()
    stream = _lib.stream_handle(torch.device(DEV))
    assert lib.kairo_bsr_stack_build(ctypes.byref(desc), 2, mem.data_ptr(), mem.numel(), ctypes.byref(st), stream) == 0
    assert st.rows_per_group == 2 and st.ngroups == (a.nbr + 1) // 2 and 0 < st.nsuper <= a.nnzb
    cfg = _lib.KairoSpmmConfig()
    wsb = ctypes.c_size_t(0)
    assert lib.kairo_bsr_spmm_stacked_workspace_size(ctypes.byref(desc), ctypes.byref(st), spec.n, ctypes.byref(cfg),
                                                     ctypes.byref(wsb)) == 0
    ws = torch.zeros(wsb.value, dtype=torch.uint8, device=DEV)
    b = p.b.to(DEV)
    c = torch.empty(spec.m, spec.n, device=DEV)
    assert lib.kairo_bsr_spmm_stacked(ctypes.byref(desc), ctypes.byref(st), b.data_ptr(), spec.n, spec.n,
                                      c.data_ptr(), spec.n, ctypes.byref(cfg), ws.data_ptr(), ws.numel(), stream) == 0
    torch.cuda.synchronize()
    assert _lib.read_workspace_error(ws) == 0
    assert rel_fro(c.cpu(), _oracle(spec, p)) <= TOL
    # four 32-row blocks per group at n_tile 256 exceed the instantiated kernels
    bad = _lib.KairoSpmmConfig()
    bad.n_tile = 256
    st4 = _lib.KairoBsrStack()
    assert lib.kairo_bsr_stack_size(ctypes.byref(desc), 4, ctypes.byref(nbytes)) == 0
    mem4 = torch.empty(nbytes.value, dtype=torch.uint8, device=DEV)
    assert lib.kairo_bsr_stack_build(ctypes.byref(desc), 4, mem4.data_ptr(), mem4.numel(), ctypes.byref(st4),
                                     stream) == 0
    assert lib.kairo_bsr_spmm_stacked(ctypes.byref(desc), ctypes.byref(st4), b.data_ptr(), spec.n, spec.n,
                                      c.data_ptr(), spec.n, ctypes.byref(bad), ws.data_ptr(), ws.numel(),
                                      stream) == _lib.NOT_SUPPORTED


@pytest.mark.slow
def test_groups_zipf_full_size_vs_rows():
    """The full-size Zipf workload (65536^2, 16x16 blocks, N = 128) through
    row groups and through the row-split schedule agree to fp32 rounding
    (the row-split result is checked against the oracle by the full-size
    tests)."""
    spec = WORKLOADS["fp16_zipf"]
    p = generate(spec, seed=0, device=DEV)
    a = bsr_from_tiles(p.tiles, p.row_ids, p.col_ids, (spec.m, spec.k))
    g = block_sparse_mm_bsr(a, p.b, config=KernelConfig(schedule="groups", group_rows=4), check=True)
    r = block_sparse_mm_bsr(a, p.b, config=KernelConfig(schedule="rows"), check=True)
    assert rel_fro(g.cpu(), r.cpu()) <= 1e-5
