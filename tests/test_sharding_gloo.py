"""The multi-GPU path's host logic, run as two gloo ranks on CPU.

Each rank shards a BSR matrix by nnz-balanced block-rows, computes its rows
(here with the CPU oracle standing in for the kernel, as the checker), and
all-gathers C.  The gathered C must equal the single-process result bit for
bit (every block-row is computed by exactly one rank, in the same order).
The failure test makes one rank raise before the collective; the other rank
must get an error from its gather within the process-group timeout instead
of waiting forever.
"""

from __future__ import annotations

import multiprocessing as mp
import os
import socket
import time
from datetime import timedelta
from pathlib import Path

import pytest
import torch

GOLDEN = Path(__file__).parent / "golden"


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _bsr_from_golden(g):
    from kairo_b200.types import BlockSparseMatrix

    perm = g["perm"]
    return BlockSparseMatrix(row_ptr=g["row_offsets"].to(torch.int32), col_idx=g["cols_sorted"].to(torch.int32),
                             blocks=g["tiles"][perm].contiguous(), shape=(g["M"], g["K"]),
                             block_size=(g["tile"], g["tile"]))


def _oracle_compute(K, N):
    from oracle import oracle

    def compute(a, B):
        out = oracle.spmm_bsr_rows(a.row_ptr, a.col_idx, a.blk_idx, a.blocks, B, a.shape[0], K,
                                   B.shape[1] if N is None else N, list(range(a.nbr)), nthreads=1)
        return out[: a.shape[0]]

    return compute


def _grid_problem(n=512):
    """A seeded 48 x 40 block grid (bs 16) in BSR order and a B with n
    columns, the same on every rank."""
    from kairo_b200.types import BlockSparseMatrix

    g = torch.Generator().manual_seed(17)
    nbr, nbc, bs = 48, 40, 16
    keep = torch.rand(nbr, nbc, generator=g) < 0.2
    keep[5] = False  # an empty block-row
    rows, cols = keep.nonzero(as_tuple=True)
    counts = torch.bincount(rows, minlength=nbr)
    row_ptr = torch.zeros(nbr + 1, dtype=torch.int32)
    row_ptr[1:] = torch.cumsum(counts, 0).to(torch.int32)
    blocks = torch.randn(rows.numel(), bs, bs, generator=g)
    B = torch.randn(nbc * bs, n, generator=g)
    a = BlockSparseMatrix(row_ptr=row_ptr, col_idx=cols.to(torch.int32), blocks=blocks, shape=(nbr * bs, nbc * bs),
                          block_size=(bs, bs))
    return a, B


def _grid_worker(rank, world, port, out_dir):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    try:
        from kairo_b200.sharding import ShardedSpmm

        a, B = _grid_problem()
        s = ShardedSpmm(a, compute=_oracle_compute(a.shape[1], None), n=B.shape[1])
        tile = s.forward(B, gather=False)
        full = s.forward(B, gather=True)
        torch.save({"tile": tile, "full": full, "grid": (s.row_groups, s.col_slices), "columns": s.columns,
                    "rows": s.shard.rows}, Path(out_dir) / f"g{rank}.pt")
    finally:
        dist.destroy_process_group()


def _worker(rank, world, port, case, out_dir, mode):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    try:
        from kairo_b200.sharding import ShardedSpmm

        g = torch.load(case, weights_only=False)
        a = _bsr_from_golden(g)
        s = ShardedSpmm(a, compute=_oracle_compute(g["K"], g["N"]))
        if mode == "fail" and rank == 1:
            raise RuntimeError("injected failure on rank 1")
        t0 = time.time()
        try:
            c = s.forward(g["B"].float(), gather=True)
            torch.save({"c": c, "bounds": s.bounds, "local_rows": s.local.shape[0]}, Path(out_dir) / f"r{rank}.pt")
        except Exception as exc:  # noqa: BLE001 - recorded for the test
            (Path(out_dir) / f"r{rank}.err").write_text(f"{type(exc).__name__}: {exc} after {time.time() - t0:.1f}s")
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(case, tmp_path, mode, world=2):
    from oracle import oracle

    oracle.build()
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(case), str(tmp_path), mode)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("a rank did not finish")
    return procs


@pytest.mark.parametrize("case", ["wl_bf16_uniform", "wl_fp16_zipf", "ragged_edges"])
def test_sharded_spmm_gather_matches_single_process(case, tmp_path):
    from oracle import oracle

    path = GOLDEN / f"{case}.pt"
    _run(path, tmp_path, "ok")
    g = torch.load(path, weights_only=False)
    a = _bsr_from_golden(g)
    full = oracle.spmm_bsr_rows(a.row_ptr, a.col_idx, None, a.blocks, g["B"].float(), g["M"], g["K"], g["N"],
                                list(range(a.nbr)), nthreads=1)[: g["M"]]
    r0 = torch.load(tmp_path / "r0.pt", weights_only=False)
    r1 = torch.load(tmp_path / "r1.pt", weights_only=False)
    assert torch.equal(r0["c"], full)
    assert torch.equal(r1["c"], full)
    b = r0["bounds"]
    assert b[0] == 0 and b[-1] == a.nbr
    rp = g["row_offsets"]
    share0 = int(rp[b[1]] - rp[b[0]])
    share1 = int(rp[b[2]] - rp[b[1]])
    assert abs(share0 - share1) <= int((rp[1:] - rp[:-1]).max()) + 1


def test_rank_failure_surfaces_as_error_not_hang(tmp_path):
    procs = _run(GOLDEN / "wl_bf16_uniform.pt", tmp_path, "fail")
    assert procs[1].exitcode != 0          # the injected failure
    assert (tmp_path / "r0.err").exists()  # rank 0's collective failed...
    assert not (tmp_path / "r0.pt").exists()
    msg = (tmp_path / "r0.err").read_text()
    seconds = float(msg.rsplit("after ", 1)[1].rstrip("s"))
    assert seconds < 60                    # ...within the process-group timeout


def test_grid_shape_and_columns():
    from kairo_b200.sharding import column_range, grid_coords, grid_shape

    assert [grid_shape(w, 1024) for w in (1, 2, 4, 8)] == [(1, 1), (1, 2), (1, 4), (2, 4)]
    assert grid_shape(8, 256) == (8, 1) and grid_shape(8, 8192) == (1, 8) and grid_shape(6, 4096) == (3, 2)
    for n, parts in ((1024, 4), (1000, 3), (300, 2), (128, 1)):
        cols = [column_range(n, parts, j) for j in range(parts)]
        assert cols[0][0] == 0 and cols[-1][1] == n
        assert all(cols[j][1] == cols[j + 1][0] for j in range(parts - 1))
        assert all(c0 % 128 == 0 for c0, _ in cols)
    assert grid_coords(5, 8, 1024) == (1, 1, 2, 4)
    # sized: A / row groups + B / column slices per rank, smallest wins
    a_b, b_b = 687_000_000, 537_000_000
    assert [grid_shape(w, 1024, a_bytes=a_b, b_bytes=b_b) for w in (1, 2, 4, 8)] == [(1, 1), (2, 1), (2, 2), (4, 2)]
    assert grid_shape(8, 1024, a_bytes=10, b_bytes=10_000) == (2, 4)        # B dominates: most slices allowed
    assert grid_shape(8, 1024, a_bytes=10_000, b_bytes=10) == (8, 1)        # A dominates: rows only


@pytest.mark.parametrize("world", [2, 4])
def test_grid_sharded_spmm_matches_single_process(world, tmp_path):
    """(row groups x column slices) shards, computed with the oracle and
    gathered, equal the single-process product bit for bit."""
    from oracle import oracle

    oracle.build()
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_grid_worker, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("a rank did not finish")
    a, B = _grid_problem()
    full = oracle.spmm_bsr_rows(a.row_ptr, a.col_idx, None, a.blocks, B, a.shape[0], a.shape[1], B.shape[1],
                                list(range(a.nbr)), nthreads=1)[: a.shape[0]]
    covered = torch.zeros_like(full, dtype=torch.int32)
    for r in range(world):
        d = torch.load(tmp_path / f"g{r}.pt", weights_only=False)
        assert d["grid"] == ((1, 2) if world == 2 else (2, 2))
        assert torch.equal(d["full"], full)
        (r0, r1), (c0, c1) = d["rows"], d["columns"]
        r1 = min(r1, full.shape[0])
        assert torch.equal(d["tile"], full[r0:r1, c0:c1])
        covered[r0:r1, c0:c1] += 1
    assert bool((covered == 1).all())
