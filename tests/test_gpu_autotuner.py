"""The autotuner's GPU timing path (kairo/ops/_autotuner.py:66-178 is the
reference's): ``best_config`` times every candidate tile and launch variant
on the device and returns the fastest, and the configuration it returns
computes the oracle's result.  ``best_kernel_config`` does the same on an
actual matrix."""

from __future__ import annotations

import pytest
import torch

from oracle import oracle
from kairo_b200 import _lib
from kairo_b200.ops import KernelConfig, TileAutotuner, block_sparse_mm_bsr, bsr_from_tiles, describe
from kairo_b200.ops._autotuner import BLACKWELL_VARIANTS, CANDIDATE_CONFIGS, GROUP_VARIANTS
from kairo_b200.workloads import WorkloadSpec, generate
from tests.conftest import rel_fro

pytestmark = pytest.mark.gpu

TOL = 1e-3


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_best_config_times_on_the_gpu_and_its_choice_matches_the_oracle(dtype):
    tuner = TileAutotuner()
    M, K, N, sp = 2048, 2048, 256, 0.9
    cfg = tuner.best_config(M, K, N, sp, dtype=dtype)
    assert cfg["tile_m"] in (16, 32, 64) and cfg["tile_k"] in (16, 32)
    assert len(tuner._cache) == 1
    assert tuner.best_config(M, K, N, sp, dtype=dtype) is cfg  # cached
    # The chosen tile and launch knobs, run on a problem of that tile size.
    spec = WorkloadSpec("t", dtype, M, K, N, cfg["tile_m"], sp)
    p = generate(spec, seed=8)
    a = bsr_from_tiles(p.tiles.cuda(), p.row_ids.cuda(), p.col_ids.cuda(), (M, K))
    kc = KernelConfig(n_tile=cfg["n_tile"], stages=cfg["stages"], row_cost=cfg["row_cost"],
                      schedule=cfg["schedule"], group_blocks=cfg["group_blocks"], ctas_per_sm=cfg["ctas_per_sm"])
    c = block_sparse_mm_bsr(a, p.b.cuda(), config=kc, check=True)
    ref = oracle.spmm_tiles(p.tiles, p.row_ids, p.col_ids, p.b, M, K, N, spec.block)
    assert rel_fro(c, ref) <= TOL


def test_every_candidate_is_timed():
    tuner = TileAutotuner()
    cands = tuner.candidates(1024, 1024, torch.float16)
    square = [c for c in CANDIDATE_CONFIGS if c.tile_m == c.tile_k]
    assert len(cands) == len(square) * len(BLACKWELL_VARIANTS) + (len(CANDIDATE_CONFIGS) - len(square))
    times = [tuner._time_config(c, 1024, 1024, 128, 0.9, torch.float16) for c in cands]
    assert all(t > 0 for t in times)
    # the library default of every tile size always runs
    assert all(t < float("inf") for c, t in zip(cands, times) if c.kernel_config() == KernelConfig())


def test_best_kernel_config_on_a_matrix():
    spec = WorkloadSpec("t", torch.bfloat16, 4096, 4096, 512, 32, 0.97)
    p = generate(spec, seed=9)
    a = bsr_from_tiles(p.tiles.cuda(), p.row_ids.cuda(), p.col_ids.cuda(), (spec.m, spec.k))
    tuner = TileAutotuner()
    timed = tuner.time_kernel_configs(a, spec.n)
    assert len(timed) == len(BLACKWELL_VARIANTS) + len(GROUP_VARIANTS)
    assert sum(kc.schedule == "groups" for kc, _ in timed) == len(GROUP_VARIANTS)
    for kc, t in timed:
        # a variant whose pipeline does not fit this block shape (e.g. 8
        # blocks of 256 columns per stage) is skipped as inf, as in the
        # reference; every other one is timed
        try:
            describe(a, spec.n, config=kc)
        except _lib.KairoError:
            assert t == float("inf")
            continue
        assert 0 < t < float("inf")
    best = tuner.best_kernel_config(a, spec.n)
    assert tuner.best_kernel_config(a, spec.n) == best  # cached
    c = block_sparse_mm_bsr(a, p.b.cuda(), config=best, check=True)
    ref = oracle.spmm_tiles(p.tiles, p.row_ids, p.col_ids, p.b, spec.m, spec.k, spec.n, spec.block)
    assert rel_fro(c, ref) <= TOL
