"""A bounded pipeline wait that runs out, on the GPU, without a fault.

Every mbarrier wait of the tcgen05 kernels is bounded: on timeout the
kernel records KAIRO_DEVERR_WAIT_TIMEOUT with the wait's site tag in the
workspace error word, stops all its roles, lets the copies it issued land,
frees its TMEM and returns, so the CUDA context stays usable.  Here the
launch knobs make that path run: a short bound (wait_kcycles, thousands of
SM cycles) and the test hook debug_hold_stage, with which the producer holds
back the arrival of its first stage until a consumer's wait has run out.
Nothing traps, faults or waits without a bound.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from oracle import oracle
from kairo_b200 import _lib
from kairo_b200.ops import KernelConfig, block_sparse_mm_bsr, bsr_from_tiles, describe
from kairo_b200.ops.spmm import _bsr_desc
from kairo_b200.workloads import WorkloadSpec, generate
from tests.conftest import rel_fro

pytestmark = pytest.mark.gpu

TOL = 1e-3
# The consumers that can see the held stage first: the MMA issuer waiting
# for it, or the epilogue waiting for the accumulator that depends on it.
HELD_SITES = (_lib.WAIT_SITE_FULL, _lib.WAIT_SITE_TMEM_FULL)


def _problem():
    spec = WorkloadSpec("t", torch.float16, 1024, 1024, 256, 32, 0.9)
    p = generate(spec, seed=3)
    a = bsr_from_tiles(p.tiles.cuda(), p.row_ids.cuda(), p.col_ids.cuda(), (spec.m, spec.k))
    ref = oracle.spmm_tiles(p.tiles, p.row_ids, p.col_ids, p.b, spec.m, spec.k, spec.n, spec.block)
    return spec, a, p.b.cuda(), ref


def test_held_stage_times_out_through_the_c_abi_and_the_workspace_recovers():
    spec, a, b, ref = _problem()
    lib = _lib.lib()
    held = KernelConfig(schedule="rows", num_ctas=8, wait_kcycles=200, debug_hold_stage=1)
    assert describe(a, spec.n, config=held)["schedule"] == "rows"
    desc = _bsr_desc(a)
    nbytes = ctypes.c_size_t(0)
    _lib.check(lib.kairo_bsr_spmm_workspace_size(ctypes.byref(desc), _lib.LAYOUT_STANDARD, spec.n,
                                                 ctypes.byref(held.to_c()), ctypes.byref(nbytes)), "size")
    ws = torch.zeros(max(nbytes.value, 1 << 20), dtype=torch.uint8, device="cuda")
    stream = _lib.stream_handle(b.device)
    c = torch.zeros(spec.m, spec.n, device="cuda")

    def launch(cfg):
        st = lib.kairo_bsr_spmm(ctypes.byref(desc), b.data_ptr(), b.stride(0), _lib.LAYOUT_STANDARD, spec.n,
                                c.data_ptr(), c.stride(0), _lib.DTYPE_F32, ctypes.byref(cfg.to_c()), ws.data_ptr(),
                                ws.numel(), stream)
        assert st == _lib.SUCCESS, lib.kairo_last_error_message()
        code = ctypes.c_uint32(0)
        _lib.check(lib.kairo_workspace_error(ws.data_ptr(), 1, ctypes.byref(code), stream), "error word")
        return int(code.value)

    code = launch(held)
    assert code & 0xFF == _lib.DEVERR_WAIT_TIMEOUT
    assert (code >> 8) & 0xFF in HELD_SITES
    # The context and the workspace are still good: a normal launch on the
    # same workspace computes C (its counter bank was zeroed by the aborted
    # launch), and so does the next one, on the other bank.
    for _ in range(2):
        assert launch(KernelConfig(schedule="rows", num_ctas=8)) == 0
        assert rel_fro(c, ref) <= TOL


def test_held_stage_raises_through_the_operator():
    spec, a, b, ref = _problem()
    cfg = KernelConfig(schedule="rows", wait_kcycles=200, debug_hold_stage=1)
    with pytest.raises(_lib.KairoDeviceError) as err:
        block_sparse_mm_bsr(a, b, config=cfg, check=True)
    assert err.value.code & 0xFF == _lib.DEVERR_WAIT_TIMEOUT
    assert (err.value.code >> 8) & 0xFF in HELD_SITES
    c = block_sparse_mm_bsr(a, b, check=True)
    assert rel_fro(c, ref) <= TOL


def test_short_wait_bound_alone_does_not_fire():
    """A short bound without the hook: normal waits end well inside it."""
    spec, a, b, ref = _problem()
    c = block_sparse_mm_bsr(a, b, config=KernelConfig(schedule="rows", wait_kcycles=20000), check=True)
    assert rel_fro(c, ref) <= TOL
