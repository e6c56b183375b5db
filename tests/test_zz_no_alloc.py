"""kairo_bsr_spmm_noalloc: the SpMM entry point that allocates nothing.

It exists for callers that cannot allocate device memory: a framework that
forbids plugins to cudaMalloc, a path that must not stall the device, or a
stateless callback with no workspace to keep alive.  Its scratch is an array
built into the library and shared by all calls on a device.  So these tests
check two calls in a row (the second sees the first one's leftovers) against
the workspace-taking entry point, and the refusal of a problem too large for
the array.  The file name sorts last, so a run that stops at the first
failure has already run every other test.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from kairo_b200 import _lib
from kairo_b200.ops import KernelConfig, bsr_from_tiles
from kairo_b200.ops.spmm import _bsr_desc
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


@pytest.mark.parametrize("spec,cfg", [
    (WorkloadSpec("t", torch.float16, 1024, 1024, 256, 32, 0.9), KernelConfig()),
    (WorkloadSpec("t", torch.bfloat16, 2048, 2048, 128, 16, 0.99, mask="zipf"), KernelConfig(num_ctas=7)),
    (WorkloadSpec("t", torch.float32, 512, 512, 64, 16, 0.8), KernelConfig()),
])
def test_noalloc_matches_workspace_entry_point_twice(spec, cfg):
    p = generate(spec, seed=5)
    a = bsr_from_tiles(p.tiles.cuda(), p.row_ids.cuda(), p.col_ids.cuda(), (spec.m, spec.k))
    b = p.b.cuda()
    ccfg = cfg.to_c()
    ref = torch.empty(spec.m, spec.n, dtype=torch.float32, device="cuda")
    _with_workspace(a, b, _lib.LAYOUT_STANDARD, spec.n, ref, _lib.DTYPE_F32, ccfg)
    for _ in range(2):
        c = torch.full((spec.m, spec.n), float("nan"), device="cuda")
        st = _noalloc(a, b, _lib.LAYOUT_STANDARD, spec.n, c, _lib.DTYPE_F32, ccfg)
        assert st == _lib.SUCCESS, _lib.lib().kairo_last_error_message()
        torch.cuda.synchronize()
        assert rel_fro(c, ref) <= TOL


def test_noalloc_refuses_problems_beyond_its_scratch():
    # One 64x64 block but 65536 columns: the split-row partial tiles of the
    # plan exceed the 32 MiB array, so the call must refuse before launching.
    tiles = torch.randn(1, 64, 64, device="cuda").to(torch.bfloat16)
    a = bsr_from_tiles(tiles, torch.zeros(1, dtype=torch.int32, device="cuda"),
                       torch.zeros(1, dtype=torch.int32, device="cuda"), (64, 64))
    n = 65536
    b = torch.zeros(64, n, dtype=torch.bfloat16, device="cuda")
    c = torch.full((64, n), 7.0, device="cuda")
    st = _noalloc(a, b, _lib.LAYOUT_STANDARD, n, c, _lib.DTYPE_F32, KernelConfig().to_c())
    assert st == _lib.NOT_SUPPORTED
    assert b"scratch" in _lib.lib().kairo_last_error_message()
    torch.cuda.synchronize()
    assert torch.all(c == 7.0)
