"""Host-side pieces of bench.py and of the result checker, on CPU: the
strict roofline arithmetic, the rule that a committed traffic capture is
used only for its own launch plan, the reference arm's BSR built on the host
by the oracle (the reference's row-sort convention), and the per-block-row
comparison the checker reports."""

from __future__ import annotations

import json

import pytest
import torch

import bench
from oracle import oracle
from kairo_b200.types import BlockSparseMatrix
from kairo_b200.workloads import WORKLOADS, block_row_errors, generate, rel_fro_chunked


def test_strict_roofline_picks_the_longer_bound_and_never_exceeds_one():
    # 1 TFLOP at 1000 TFLOP/s = 1 ms; 1 GB at 1000 GB/s = 1 ms + a hair
    r = bench.strict_roofline(1e12, 1.0e9, 2.0, 1000.0, 1000.0)
    assert r["bound"] == "tensor" and r["unit"] == "TFLOP/s"
    assert r["frac"] == pytest.approx(0.5) and r["achieved"] == pytest.approx(500.0)
    r = bench.strict_roofline(1e9, 4e9, 2.0, 1000.0, 1000.0)
    assert r["bound"] == "hbm" and r["unit"] == "GB/s" and r["frac"] == pytest.approx(2.0)  # 4 ms of bytes in 2 ms
    r = bench.strict_roofline(1e9, 4e9, 8.0, 1000.0, 1000.0, compute_bound="fp32")
    assert r["bound"] == "hbm" and r["frac"] == pytest.approx(0.5)
    assert bench.strict_roofline(4e12, 1e9, 8.0, 1000.0, 1000.0, compute_bound="fp32")["bound"] == "fp32"


def test_traffic_is_used_only_for_the_captured_plan(tmp_path, monkeypatch):
    plan = {"kernel": "tcgen05", "schedule": "rows", "grid": 296, "n_tile": 256, "stages": 3, "group_blocks": 2,
            "rows": 8, "launches": 1, "workspace_bytes": 1}
    (tmp_path / "profiles").mkdir()
    (tmp_path / "profiles" / "traffic_w.txt").write_text(
        "header line\nn_gpus: 1\nplan: " + json.dumps({k: plan[k] for k in ("kernel", "schedule", "grid", "n_tile",
                                                                          "stages", "group_blocks", "rows")})
        + "\ndram_bytes_per_launch: 123456\n")
    monkeypatch.setattr(bench, "ROOT", tmp_path)
    assert bench.load_traffic("w", 1, plan) == 123456.0
    assert bench.load_traffic("w", 2, plan) is None                      # another GPU count
    assert bench.load_traffic("w", 1, dict(plan, grid=148)) is None      # another launch plan
    assert bench.load_traffic("other", 1, plan) is None                  # no capture


@pytest.mark.parametrize("name", ["fp16_uniform", "fp16_zipf", "bf16_linear"])
def test_reference_arm_bsr_is_the_reference_convention(name):
    spec = WORKLOADS[name].scaled(1024, 2048, 128) if name != "fp16_zipf" else WORKLOADS[name].scaled(2048, 2048, 64)
    p = generate(spec, seed=1)
    g = torch.Generator().manual_seed(2)
    perm = torch.randperm(p.mask.nnz, generator=g)   # an unsorted tile list
    from kairo_b200.types import SparseMask
    mask = SparseMask(p.mask.indices[:, perm], p.mask.values[perm], p.mask.dense_shape, p.mask.sparsity_ratio)
    q = type(p)(spec=spec, mask=mask, tiles=p.tiles[perm].contiguous(), b=p.b)
    row_ptr, col_idx, blocks, b = bench.host_bsr_from_coo(q)
    rows = mask.indices[0]
    order = torch.argsort(rows, stable=True)                 # sparse_embedding.py:55
    assert torch.equal(col_idx.long(), mask.indices[1][order])
    assert torch.equal(blocks, q.tiles[order])
    counts = torch.bincount(rows, minlength=spec.nbr)
    assert torch.equal(row_ptr.long(), torch.cat([torch.zeros(1, dtype=torch.long), counts.cumsum(0)]))
    # the checker on exactly the oracle's product reports zero, and finds one changed element
    a = BlockSparseMatrix(row_ptr=row_ptr, col_idx=col_idx, blocks=blocks, shape=(spec.m, spec.k),
                          block_size=(spec.block, spec.block))
    linear = spec.layout == "linear"
    ref = oracle.spmm_tiles(q.tiles, q.row_ids, q.col_ids, b, spec.m, spec.k, spec.n, spec.block)
    out = ref.t().contiguous().to(spec.out_dtype) if linear else ref.clone()
    assert bench.check_output(a, q.b, out, linear)["max_block_row_rel_err"] == 0.0
    out.view(-1)[17] += 100.0
    assert bench.check_output(a, q.b, out, linear)["max_block_row_rel_err"] > 1e-3


def test_block_row_errors_localise_one_bad_row():
    c = torch.randn(4096, 64)
    ref = c.clone()
    ref[992:1024] *= 1.01             # block-row 31 of 32-row blocks, 1 % off
    rows = block_row_errors(c, ref, 32, chunk_rows=512)
    assert rows.shape == (128,)
    assert int(torch.argmax(rows)) == 31 and float(rows[31]) == pytest.approx(0.01 / 1.01, rel=1e-3)
    assert float(rows[30]) == 0.0
    # the whole-matrix error of the same difference is far below the bar
    assert rel_fro_chunked(c, ref, chunk_rows=700) < 1e-3 < float(rows.max())


def test_workload_overrides_shape_and_sparsity():
    """--shape and --sparsity derive a named variant of a workload (its own
    name, so a committed traffic capture of the original never applies)."""
    import argparse

    args = argparse.Namespace(workload="fp16_zipf", shape="", sparsity=None)
    assert bench.workload_spec(args) == WORKLOADS["fp16_zipf"]
    args = argparse.Namespace(workload="fp16_zipf", shape="8192x8192x128", sparsity=0.999)
    spec = bench.workload_spec(args)
    assert (spec.m, spec.k, spec.n, spec.sparsity, spec.mask) == (8192, 8192, 128, 0.999, "zipf")
    assert spec.name != WORKLOADS["fp16_zipf"].name and "sparsity0.999" in spec.name
    assert spec.nnzb == max(1, int(spec.nbr * spec.nbc * (1 - 0.999)))
