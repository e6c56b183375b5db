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
        out = oracle.spmm_bsr_rows(a.row_ptr, a.col_idx, a.blk_idx, a.blocks, B, a.shape[0], K, N,
                                   list(range(a.nbr)), nthreads=1)
        return out[: a.shape[0]]

    return compute


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
