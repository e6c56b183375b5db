"""Host-side behaviour of the reference-facing interface (no GPU needed).

Ports the reference's non-CUDA SpMM tests (tests/ops/test_spmm_ops.py) that
exercise the interface contract: argument errors, the empty-mask rule, the
autotuner contract, and the SparseMask type.  Numerical tests of the kernels
are in test_gpu_parity.py.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from kairo_b200 import _C
from kairo_b200.ops import (
    KernelConfig,
    TileAutotuner,
    TileConfig,
    block_sparse_mm,
    cuda_ext_available,
)
from kairo_b200.ops._autotuner import CANDIDATE_CONFIGS, DEFAULT_CONFIG, _cache_key
from kairo_b200.types import BlockSparseMatrix, SparseMask
from kairo_b200.workloads import (
    WORKLOADS,
    WorkloadSpec,
    canonical_bytes,
    flops,
    generate,
    strict_bytes,
    zipf_counts,
)

GOLDEN = Path(__file__).parent / "golden"


def _mask(nbr, nbc, sparsity, seed=42):
    torch.manual_seed(seed)
    total = nbr * nbc
    nnz = max(1, int(total * (1.0 - sparsity)))
    perm = torch.randperm(total)[:nnz]
    rows, cols = perm // nbc, perm % nbc
    idx = torch.argsort(rows, stable=True)
    return SparseMask(torch.stack([rows[idx], cols[idx]]).to(torch.int64), torch.ones(nnz), (nbr, nbc), sparsity)


# --------------------------------------------------------------- SparseMask

def test_sparse_mask_to_dense_and_nnz():
    m = SparseMask(torch.tensor([[0, 1], [1, 0]]), torch.ones(2), (2, 3), 4 / 6)
    d = m.to_dense()
    assert d.shape == (2, 3)
    assert d[0, 1] == 1 and d[1, 0] == 1 and d.sum() == 2
    assert m.nnz == 2
    assert m.device.type == "cpu"


def test_sparse_mask_is_frozen():
    m = SparseMask(torch.zeros(2, 0, dtype=torch.int64), torch.zeros(0), (1, 1), 1.0)
    with pytest.raises(Exception):
        m.nnz = 3  # type: ignore[misc]


# --------------------------------------------------------------- BlockSparseMatrix

def test_block_sparse_matrix_validation():
    rp = torch.tensor([0, 1, 1], dtype=torch.int32)
    ci = torch.tensor([0], dtype=torch.int32)
    blocks = torch.zeros(1, 16, 16)
    a = BlockSparseMatrix(rp, ci, blocks, (32, 16), (16, 16))
    assert a.nbr == 2 and a.nbc == 1 and a.nnzb == 1
    assert a.sparsity == pytest.approx(0.5)
    with pytest.raises(ValueError, match="row_ptr must have"):
        BlockSparseMatrix(rp[:2], ci, blocks, (32, 16), (16, 16))
    with pytest.raises(ValueError, match="int32"):
        BlockSparseMatrix(rp.long(), ci, blocks, (32, 16), (16, 16))
    with pytest.raises(ValueError, match="blocks must be"):
        BlockSparseMatrix(rp, ci, torch.zeros(1, 16, 8), (32, 16), (16, 16))
    with pytest.raises(ValueError, match="fewer stored blocks"):
        BlockSparseMatrix(rp, ci, torch.zeros(0, 16, 16), (32, 16), (16, 16))


def test_kernel_config_validation():
    assert KernelConfig().to_c().kernel == 0
    assert KernelConfig(kernel="tcgen05", n_tile=256, group_blocks=4).to_c().group_blocks == 4
    with pytest.raises(ValueError):
        KernelConfig(kernel="triton")
    with pytest.raises(ValueError):
        KernelConfig(n_tile=512)
    with pytest.raises(ValueError):
        KernelConfig(stages=-1)
    with pytest.raises(ValueError):
        KernelConfig(group_blocks=33)


# --------------------------------------------------------------- operator contract

def test_dimension_mismatch_raises():
    """tests/ops/test_spmm_ops.py:186-191: checked before anything else."""
    A = torch.randn(32, 32)
    B = torch.randn(16, 16)
    with pytest.raises(ValueError, match="Inner dimensions must match"):
        block_sparse_mm(A, B, _mask(2, 2, 0.0), tile_size=16)


def test_cpu_tensors_are_rejected_not_computed():
    """No CPU implementation: CPU inputs raise instead of silently falling back."""
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        block_sparse_mm(torch.randn(32, 32), torch.randn(32, 16), _mask(2, 2, 0.5), tile_size=16)


@pytest.mark.parametrize(
    "kwargs,msg",
    [
        ({"A_tiles": torch.zeros(2, 16, 16).transpose(1, 2)}, "A_tiles must be contiguous"),
        ({"tile_row_ids": torch.zeros(2, dtype=torch.int64)}, "tile_row_ids must be int32"),
        ({"tile_col_ids": torch.zeros(2, dtype=torch.int64)}, "tile_col_ids must be int32"),
        ({"M": 0}, "dimensions must be positive"),
        ({}, "A_tiles must be on CUDA"),
    ],
)
def test_acc_spmm_forward_argument_checks(kwargs, msg):
    """bindings.cpp:92-100 and acc_spmm_kernel.cu:166-167: same checks, same messages."""
    args = {"A_tiles": torch.zeros(2, 16, 16), "tile_row_ids": torch.zeros(2, dtype=torch.int32),
            "tile_col_ids": torch.zeros(2, dtype=torch.int32), "B": torch.zeros(32, 16), "M": 32, "K": 32, "N": 16,
            "num_tiles": 2, "tile_m": 16, "tile_k": 16}
    args.update(kwargs)
    with pytest.raises(RuntimeError, match=msg):
        _C.acc_spmm_forward(**args)


def test_cuda_ext_available_reports_library():
    assert cuda_ext_available() is True


# --------------------------------------------------------------- autotuner contract

def test_autotuner_returns_valid_config():
    """tests/ops/test_spmm_ops.py:199-228 (keys, ranges, cache, clear, CPU default)."""
    at = TileAutotuner()
    cfg = at.best_config(M=256, K=256, N=128, sparsity=0.5)
    assert {"tile_m", "tile_n", "tile_k"} <= set(cfg)
    assert cfg["tile_m"] in (16, 32, 64)
    assert cfg["tile_k"] in (16, 32)
    assert at.best_config(M=256, K=256, N=128, sparsity=0.5) == cfg
    assert len(at._cache) > 0
    at.clear_cache()
    assert len(at._cache) == 0
    assert at.best_config(M=64, K=64, N=32, sparsity=0.5)["tile_m"] >= 16


def test_autotuner_blackwell_keys_and_cache_key():
    assert DEFAULT_CONFIG == CANDIDATE_CONFIGS[0] == TileConfig(16, 16, 16)
    cfg = TileAutotuner().best_config(4096, 4096, 256, 0.9, dtype=torch.float16)
    assert {"n_tile", "stages", "row_cost"} <= set(cfg)
    assert _cache_key(100, 600, 3000, 0.94) == "128_2048_4096_0.9"
    assert _cache_key(100, 600, 3000, 0.94, torch.bfloat16).endswith("_bfloat16")
    with pytest.raises(ValueError):
        TileConfig(16, 16, 16, n_tile=64)


# --------------------------------------------------------------- workloads

def test_uniform_mask_follows_reference_generator():
    """The uniform mask draws match the reference test generator recorded in
    the golden fixture (tests/ops/test_spmm_ops.py:21-44, seed 42)."""
    g = torch.load(GOLDEN / "ref_sparse95.pt", weights_only=False)
    m = _mask(4, 4, 0.95)
    assert torch.equal(m.indices, g["mask_indices"])


def test_zipf_counts_properties():
    c = zipf_counts(4096, 4096, 167772, seed=0)
    assert c.sum() == 167772
    assert c.max() == 4096 and (c <= 4096).all() and (c >= 0).all()
    assert (c == 4096).sum() == 29
    assert np.sort(c)[-10:].sum() / c.sum() > 0.2
    assert np.array_equal(c, zipf_counts(4096, 4096, 167772, seed=0))


def test_generated_problem_shapes_and_edge_zeroing():
    p = generate(WorkloadSpec("t", torch.float32, 40, 56, 24, 16, 0.3), seed=1)
    assert p.tiles.shape[1:] == (16, 16)
    r = p.mask.indices[0]
    c = p.mask.indices[1]
    assert torch.all(r[1:] >= r[:-1])  # row-sorted
    for t in range(p.mask.nnz):
        rr = int(r[t]) * 16
        cc = int(c[t]) * 16
        tile = p.tiles[t]
        if rr + 16 > 40:
            assert torch.all(tile[40 - rr:] == 0)
        if cc + 16 > 56:
            assert torch.all(tile[:, 56 - cc:] == 0)


def test_magnitude_mask_keeps_largest_blocks():
    spec = WorkloadSpec("t", torch.bfloat16, 256, 512, 16, 64, 0.75, mask="magnitude", layout="linear")
    p = generate(spec, seed=3)
    assert p.mask.nnz == spec.nnzb == 8
    flat = p.mask.indices[0] * spec.nbc + p.mask.indices[1]
    assert torch.all(flat[1:] > flat[:-1])  # kept indices sorted (topology.py:95-96 convention)
    assert p.b.shape == (16, 512)


def test_accounting_matches_definitions():
    spec = WORKLOADS["fp16_uniform"]
    assert spec.nnzb == 13107
    assert flops(spec) == pytest.approx(2 * 13107 * 32 * 32 * 512)
    canon = 13107 * 32 * 32 * 2 + (13107 + 512 + 1) * 4 + 13107 * 32 * 512 * 2 + 16384 * 512 * 4
    assert canonical_bytes(spec) == pytest.approx(canon)
    strict = canon - 13107 * 32 * 512 * 2 + 16384 * 512 * 2
    assert strict_bytes(spec) == pytest.approx(strict)
    assert WORKLOADS["bf16_uniform"].nnzb == 335544
    assert WORKLOADS["fp16_zipf"].nnzb == 167772
    assert WORKLOADS["bf16_linear"].nnzb == 13107
    assert WORKLOADS["fp32_uniform"].nnzb == 6553


def test_new_launch_knobs_are_validated_and_reach_the_c_struct():
    from kairo_b200.ops import KernelConfig

    c = KernelConfig(ctas_per_sm=2, wait_kcycles=500, debug_hold_stage=1).to_c()
    assert (c.ctas_per_sm, c.wait_kcycles, c.debug_hold_stage) == (2, 500, 1)
    with pytest.raises(ValueError):
        KernelConfig(ctas_per_sm=5)
    with pytest.raises(ValueError):
        KernelConfig(debug_hold_stage=2)
    with pytest.raises(ValueError):
        KernelConfig(wait_kcycles=-1)


def test_autotuner_candidates_and_key():
    import torch as _t
    from kairo_b200.ops._autotuner import BLACKWELL_VARIANTS, CANDIDATE_CONFIGS, TileAutotuner, _cache_key

    tuner = TileAutotuner()
    square = [c for c in CANDIDATE_CONFIGS if c.tile_m == c.tile_k]
    cands = tuner.candidates(1024, 1024, _t.bfloat16)
    assert len(cands) == len(square) * len(BLACKWELL_VARIANTS) + len(CANDIDATE_CONFIGS) - len(square)
    assert all(c.tile_m == c.tile_k or (c.n_tile, c.schedule, c.ctas_per_sm) == (0, "auto", 0) for c in cands)
    assert len(tuner.candidates(1024, 1024, _t.float32)) == len(CANDIDATE_CONFIGS)
    assert {c.tile_m for c in tuner.candidates(1024, 1024, _t.float16, block=32)} == {32}
    # the reference's 4-argument key is unchanged; dtype and block are appended
    assert _cache_key(256, 256, 128, 0.5) == "512_512_128_0.5"
    assert _cache_key(256, 256, 128, 0.5, _t.bfloat16, 32) == "512_512_128_0.5_bfloat16_b32"


def test_row_group_knobs_and_choice_without_a_device(monkeypatch):
    """Row groups: the knobs are validated, the stack descriptor has the C
    layout, and the schedule choice is made on the host (AUTO leaves them
    off unless switched on; a non-skewed matrix never builds them; the
    LINEAR layout refuses an explicit request)."""
    import ctypes

    from kairo_b200 import _lib
    from kairo_b200.ops import KernelConfig
    from kairo_b200.ops import spmm as spmm_mod

    for r in (0, 2, 4, 8):
        assert KernelConfig(schedule="groups", group_rows=r).to_c().schedule == _lib.SCHEDULE_AUTO
    for bad in (1, 3, 16):
        with pytest.raises(ValueError):
            KernelConfig(group_rows=bad)
    assert ctypes.sizeof(_lib.KairoBsrStack) == 56

    nbr, bs = 64, 16
    counts = torch.full((nbr,), 3, dtype=torch.int32)
    row_ptr = torch.cat([torch.zeros(1, dtype=torch.int32), torch.cumsum(counts, 0).to(torch.int32)])
    nnzb = int(row_ptr[-1])
    a = BlockSparseMatrix(row_ptr=row_ptr, col_idx=torch.arange(nnzb, dtype=torch.int32) % nbr,
                          blocks=torch.zeros(nnzb, bs, bs, dtype=torch.float16), shape=(nbr * bs, nbr * bs),
                          block_size=(bs, bs), max_row_blocks=3)
    assert spmm_mod._row_groups_for(a, _lib.LAYOUT_STANDARD, None) is None
    monkeypatch.setattr(spmm_mod, "_GROUPS_AUTO", True)
    assert spmm_mod._row_groups_for(a, _lib.LAYOUT_STANDARD, None) is None  # rows of equal length
    assert spmm_mod._row_groups_for(a, _lib.LAYOUT_STANDARD, KernelConfig(schedule="rows")) is None
    with pytest.raises(ValueError):
        spmm_mod._row_groups_for(a, _lib.LAYOUT_LINEAR, KernelConfig(schedule="groups"))
