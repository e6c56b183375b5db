"""kairo_bsr_spmm_noalloc: the SpMM entry point that allocates nothing.

It exists for callers that cannot allocate device memory: a framework that
forbids plugins to cudaMalloc, a path that must not stall the device, or a
stateless callback with no workspace to keep alive.  Its scratch is an array
built into the library and shared by all calls on a device, which keeps the
last call's contents.  So these tests run two calls in a row (the second
sees the first one's leftovers: split-row partial tiles, the split-bf16
path's derived operands, the band schedule's column order) and check both
against the workspace-taking entry point and against the CPU oracle.  They
also read a device error through kairo_noalloc_error (an out-of-range
block column, which the kernels bound-check: no access goes out of range)
and check the refusal of a problem too large for the array.  The file name
sorts last, so a run that stops at the first failure has already run every
other test.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from oracle import oracle
from kairo_b200 import _lib
from kairo_b200.ops import KernelConfig, bsr_from_tiles, describe
from kairo_b200.ops.spmm import _bsr_desc
from kairo_b200.types import BlockSparseMatrix
from kairo_b200.workloads import WorkloadSpec, generate
from tests.conftest import rel_fro

pytestmark = pytest.mark.gpu

TOL = 1e-3  # the relative Frobenius bar of the other SpMM tests


def _with_workspace(a, b, layout, n, c, c_dtype, cfg):
    lib = _lib.lib()
    desc = _bsr_desc(a)
    nbytes = ctypes.c_size_t(0)
    _lib.check(lib.kairo_bsr_spmm_workspace_size(ctypes.byref(desc), layout, n, ctypes.byref(cfg),
                                                 ctypes.byref(nbytes)), "workspace size")
    ws = torch.zeros(nbytes.value, dtype=torch.uint8, device=b.device)
    _lib.check(lib.kairo_bsr_spmm(ctypes.byref(desc), b.data_ptr(), b.stride(0), layout, n, c.data_ptr(),
                                  c.stride(0), c_dtype, ctypes.byref(cfg), ws.data_ptr(), ws.numel(),
                                  _lib.stream_handle(b.device)), "kairo_bsr_spmm")


def _noalloc(a, b, layout, n, c, c_dtype, cfg) -> int:
    desc = _bsr_desc(a)
    return _lib.lib().kairo_bsr_spmm_noalloc(ctypes.byref(desc), b.data_ptr(), b.stride(0), layout, n,
                                             c.data_ptr(), c.stride(0), c_dtype, ctypes.byref(cfg),
                                             _lib.stream_handle(b.device))


def _noalloc_error(clear: bool = True) -> int:
    code = ctypes.c_uint32(0xFFFFFFFF)
    _lib.check(_lib.lib().kairo_noalloc_error(1 if clear else 0, ctypes.byref(code),
                                              _lib.stream_handle(torch.device("cuda"))), "kairo_noalloc_error")
    return int(code.value)


CASES = [
    # fp16 32x32 blocks, default plan
    (WorkloadSpec("t", torch.float16, 1024, 1024, 256, 32, 0.9), KernelConfig(), None),
    # Zipf rows cut over 7 CTAs: split-row partial tiles in the scratch
    (WorkloadSpec("t", torch.bfloat16, 2048, 2048, 128, 16, 0.99, mask="zipf"),
     KernelConfig(schedule="rows", num_ctas=7), "rows"),
    # the band schedule: its per-launch column order lives in the scratch
    (WorkloadSpec("t", torch.bfloat16, 1024, 2048, 256, 32, 0.8), KernelConfig(schedule="bands"), "bands"),
    # fp32 on the CUDA cores
    (WorkloadSpec("t", torch.float32, 512, 512, 64, 16, 0.8), KernelConfig(), None),
    # fp32 through the split-bf16 path: the derived bf16 blocks and B live in the scratch
    (WorkloadSpec("t", torch.float32, 512, 768, 200, 16, 0.8), KernelConfig(kernel="split_bf16"), None),
]


@pytest.mark.parametrize("spec,cfg,schedule", CASES)
def test_noalloc_matches_workspace_entry_point_and_oracle_twice(spec, cfg, schedule):
    p = generate(spec, seed=5)
    a = bsr_from_tiles(p.tiles.cuda(), p.row_ids.cuda(), p.col_ids.cuda(), (spec.m, spec.k))
    if schedule is not None:
        assert describe(a, spec.n, config=cfg)["schedule"] == schedule
    b = p.b.cuda()
    ccfg = cfg.to_c()
    ref = torch.empty(spec.m, spec.n, dtype=torch.float32, device="cuda")
    _with_workspace(a, b, _lib.LAYOUT_STANDARD, spec.n, ref, _lib.DTYPE_F32, ccfg)
    expect = oracle.spmm_tiles(p.tiles, p.row_ids, p.col_ids, p.b, spec.m, spec.k, spec.n, spec.block)
    assert rel_fro(ref, expect) <= TOL
    for _ in range(2):
        c = torch.full((spec.m, spec.n), float("nan"), device="cuda")
        st = _noalloc(a, b, _lib.LAYOUT_STANDARD, spec.n, c, _lib.DTYPE_F32, ccfg)
        assert st == _lib.SUCCESS, _lib.lib().kairo_last_error_message()
        assert _noalloc_error() == 0
        assert rel_fro(c, ref) <= TOL
        assert rel_fro(c, expect) <= TOL


def test_noalloc_reports_a_device_error_then_recovers():
    """An out-of-range block column is caught by the kernel's bounds check
    (the load uses column 0 instead) and recorded in the scratch's error
    word; kairo_noalloc_error reads it, and the next clean call reports 0."""
    spec = WorkloadSpec("t", torch.float16, 512, 512, 128, 32, 0.8)
    p = generate(spec, seed=6)
    a = bsr_from_tiles(p.tiles.cuda(), p.row_ids.cuda(), p.col_ids.cuda(), (spec.m, spec.k))
    bad_cols = a.col_idx.clone()
    bad_cols[3] = spec.nbc + 5
    bad = BlockSparseMatrix(row_ptr=a.row_ptr, col_idx=bad_cols, blocks=a.blocks, shape=a.shape,
                            block_size=a.block_size, blk_idx=a.blk_idx, max_row_blocks=a.max_row_blocks)
    b = p.b.cuda()
    c = torch.empty(spec.m, spec.n, device="cuda")
    cfg = KernelConfig(schedule="rows").to_c()
    assert _noalloc(bad, b, _lib.LAYOUT_STANDARD, spec.n, c, _lib.DTYPE_F32, cfg) == _lib.SUCCESS
    code = _noalloc_error(clear=False)
    assert code & 0xFF == _lib.DEVERR_BAD_INDEX
    assert _noalloc_error(clear=True) == code   # read again, then cleared
    assert _noalloc_error() == 0
    assert _noalloc(a, b, _lib.LAYOUT_STANDARD, spec.n, c, _lib.DTYPE_F32, cfg) == _lib.SUCCESS
    assert _noalloc_error() == 0
    expect = oracle.spmm_tiles(p.tiles, p.row_ids, p.col_ids, p.b, spec.m, spec.k, spec.n, spec.block)
    assert rel_fro(c, expect) <= TOL


def test_noalloc_refuses_problems_beyond_its_scratch():
    # One 64x64 block but 65536 columns: the split-row partial tiles of the
    # plan exceed the 32 MiB array, so the call must refuse before launching.
    tiles = torch.randn(1, 64, 64, device="cuda").to(torch.bfloat16)
    a = bsr_from_tiles(tiles, torch.zeros(1, dtype=torch.int32, device="cuda"),
                       torch.zeros(1, dtype=torch.int32, device="cuda"), (64, 64))
    n = 65536
    b = torch.zeros(64, n, dtype=torch.bfloat16, device="cuda")
    c = torch.full((64, n), 7.0, device="cuda")
    st = _noalloc(a, b, _lib.LAYOUT_STANDARD, n, c, _lib.DTYPE_F32, KernelConfig(schedule="rows").to_c())
    assert st == _lib.NOT_SUPPORTED
    assert b"scratch" in _lib.lib().kairo_last_error_message()
    torch.cuda.synchronize()
    assert torch.all(c == 7.0)
