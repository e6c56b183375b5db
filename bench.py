"""Benchmark of the B200 BSR SpMM (C = A_bsr @ B).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload NAME] [--gather]

One process per GPU (torchrun for N > 1).  The ranks form a grid of
nnz-balanced block-row groups x column slices of B and C (``--rows``: block-row
ranges only, B replicated); no collective runs on the compute path.  Every
rank generates the same seeded workload on its device and keeps its own
shard.  A step is one SpMM launch over the local shard.  It is timed with CUDA
events on the launching stream.  The L2 is flushed before every step by
writing a 256 MiB buffer, which is not timed.  The job's time is the max over
ranks.  Rank 0 prints one JSON line.

The default workload is ``bf16_uniform``: A is 262144 x 262144 bf16 with
32x32 blocks and 99.5 % block sparsity, B is 262144 x 1024, and C is fp32.
It is the configuration defined at 1, 2, 4 and 8 GPUs, so per-N values are
comparable (strong scaling: the total work is fixed).

``--impl reference`` times the CPU restatement of the reference's SpMM path
(oracle/, multi-threaded) on rank 0 over a bounded sample of the same
workload.  Other ranks exit without work.
"""

from __future__ import annotations

import argparse
import dataclasses
import csv
import io
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from kairo_b200.workloads import WORKLOADS, canonical_bytes, flops, generate, strict_bytes  # noqa: E402

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def log(*a) -> None:
    print(*a, file=sys.stderr, flush=True)


def measured_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except Exception:  # noqa: BLE001
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def dist_env() -> tuple[int, int, int]:
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during a region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: torch.device) -> None:
        # nvidia-smi numbers GPUs physically; select ours by UUID.
        try:
            self.sel = ["-i", "GPU-" + str(torch.cuda.get_device_properties(device).uuid)]
        except Exception:  # noqa: BLE001
            self.sel = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "10", *self.sel], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self) -> dict:
        sms, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for row in csv.reader(io.StringIO(getattr(self, "out", "") or "")):
            if len(row) < 9:
                continue
            try:
                sms.append(float(row[1]))
                maxes.append(float(row[2]))
            except ValueError:
                continue
            for name, val in zip(names, row[5:9]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        if not sms:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxes), "reasons": sorted(reasons),
                "samples": len(sms)}


def l2_gather_peak(flush: torch.Tensor) -> float | None:
    """L2 -> SM bulk-copy ceiling of this GPU in GB/s (kairo_gather_probe on
    a 32 MiB, L2-resident slice; 16 KiB copies, the size of a gathered
    panel), measured live.  None if the probe fails."""
    import ctypes

    from kairo_b200 import _lib

    out = ctypes.c_double(0.0)
    st = _lib.lib().kairo_gather_probe(flush.data_ptr(), 32 << 20, 16384, 400, ctypes.byref(out),
                                       _lib.stream_handle(flush.device))
    return out.value if st == 0 else None


def load_traffic(workload: str, n_gpus: int, plan: dict) -> float | None:
    """DRAM bytes per launch of the SpMM kernel, from the committed ncu
    summary profiles/traffic_<workload>.txt, but only when that capture was
    taken of this very launch: the same number of GPUs and the same launch
    plan (kernel, schedule, grid, n_tile, stages, group_blocks, rows), both
    recorded in the file.  Anything else returns None: traffic is not
    scaled from another shape."""
    p = ROOT / "profiles" / f"traffic_{workload}.txt"
    if not p.exists():
        return None
    fields = {}
    for line in p.read_text().splitlines():
        if ":" in line:
            key, val = line.split(":", 1)
            fields[key.strip()] = val.strip()
    try:
        cap_plan = json.loads(fields.get("plan", "null"))
        if int(fields.get("n_gpus", "0")) != n_gpus or not isinstance(cap_plan, dict):
            return None
        keys = ("kernel", "schedule", "grid", "n_tile", "stages", "group_blocks", "rows")
        if any(cap_plan.get(k) != plan.get(k) for k in keys):
            return None
        return float(fields["dram_bytes_per_launch"])
    except (KeyError, ValueError):
        return None


def compute_peak(spec, plan: dict, peaks: dict, peak_kind: str) -> tuple[float, str]:
    """The arithmetic peak (TFLOP/s) of the kernel that runs: the measured
    dense bf16 tensor-core figure (burst: one kernel timed alone) for the
    tcgen05 kernels; for the fp32 CUDA-core kernel the nominal fp32 FMA peak
    of the device (2 FLOP x 128 lanes x SMs x max SM clock), since no
    measured figure exists for it."""
    if plan.get("kernel") in ("tcgen05", "split_bf16"):
        return float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])), peak_kind
    props = torch.cuda.get_device_properties(torch.cuda.current_device())
    mhz = float(peaks.get("sm_max_mhz", 1965.0))
    return 2.0 * 128 * props.multi_processor_count * mhz * 1e6 / 1e12, "nominal fp32 CUDA-core peak"


def strict_roofline(flop: float, strict: float, ms: float, tensor_tflops: float, hbm_gbs: float,
                    compute_bound: str = "tensor") -> dict:
    """Roofline fraction that cannot exceed 1 by construction: the bound is
    whichever of FLOP / arithmetic peak and strict bytes / HBM bandwidth is
    the longer, and the fraction is that time over the measured kernel time.
    ``compute_bound`` names the arithmetic unit ("tensor", or "fp32" for
    the CUDA-core kernel)."""
    t_flop = flop / (tensor_tflops * 1e12)
    t_mem = strict / (hbm_gbs * 1e9)
    t = ms / 1e3
    if t_flop >= t_mem:
        return {"bound": compute_bound, "achieved": flop / t / 1e12, "peak": tensor_tflops, "unit": "TFLOP/s",
                "frac": t_flop / t, "t_roof_ms": t_flop * 1e3, "strict_bytes": strict, "flop": flop}
    return {"bound": "hbm", "achieved": strict / t / 1e9, "peak": hbm_gbs, "unit": "GB/s", "frac": t_mem / t,
            "t_roof_ms": t_mem * 1e3, "strict_bytes": strict, "flop": flop}


def check_output(a, b, out, linear: bool) -> dict:
    """Compares the whole result of the timed launches with the oracle (the
    reference's arithmetic on fp32-widened inputs) over every block-row of
    this rank's shard: relative Frobenius error of the whole shard and the
    largest relative error of one block-row.  A bf16 result is compared with
    the oracle rounded to bf16.  The checker, run after the timed region."""
    from oracle import oracle
    from kairo_b200.workloads import block_row_errors, rel_fro_chunked

    t0 = time.perf_counter()
    m, k = a.shape
    bh = b.cpu()
    if linear:
        bh = bh.t().contiguous()  # the shard's X rows (n x K) as B (K x n)
    n = bh.shape[1]
    ref = oracle.spmm_bsr_rows(a.row_ptr.cpu(), a.col_idx.cpu(), None if a.blk_idx is None else a.blk_idx.cpu(),
                               a.blocks.cpu(), bh, m, k, n, list(range(a.nbr)))[:m]
    got = out.cpu()
    if linear:
        got = got.t()
    if got.dtype != torch.float32:
        ref = ref.to(got.dtype).float()
        got = got.float()
    err = rel_fro_chunked(got, ref)
    rows = block_row_errors(got, ref, a.block_size[0])
    return {"rel_err": err, "max_block_row_rel_err": float(rows.max()) if rows.numel() else 0.0,
            "block_rows": int(a.nbr), "tolerance": 1e-3, "seconds": time.perf_counter() - t0,
            "oracle_threads": oracle.num_threads(),
            "against": "oracle (reference arithmetic, fp32-widened inputs)" +
                       ("; bf16 result vs oracle rounded to bf16" if out.dtype != torch.float32 else "")}


def workload_spec(args):
    spec = WORKLOADS[args.workload]
    if args.shape:
        m, k, n = (int(x) for x in args.shape.lower().split("x"))
        spec = spec.scaled(m, k, n)
    if args.sparsity is not None:
        spec = dataclasses.replace(spec, name=f"{spec.name}@sparsity{args.sparsity}", sparsity=args.sparsity)
    return spec


# ---------------------------------------------------------------- CPU sample

def cpu_sample(problem, bsr_host, target_s: float, nthreads: int = 0):
    """Times the oracle (the reference's CPU algorithm, multi-threaded) on the
    first block-rows of the workload, sized for about ``target_s`` seconds.
    Returns (TFLOP/s, seconds, description)."""
    from oracle import oracle

    row_ptr, col_idx, blocks, b = bsr_host
    spec = problem.spec
    nbr = row_ptr.numel() - 1
    threads = nthreads or oracle.num_threads()
    # calibrate on a few rows
    rows = list(range(min(nbr, max(threads, 8))))
    t0 = time.perf_counter()
    oracle.spmm_bsr_rows(row_ptr, col_idx, None, blocks, b, spec.m, spec.k, spec.n, rows, nthreads=threads)
    dt = max(time.perf_counter() - t0, 1e-4)
    per_row = dt / len(rows)
    nrows = int(min(nbr, max(len(rows), target_s / per_row)))
    rows = list(range(nrows))
    t0 = time.perf_counter()
    oracle.spmm_bsr_rows(row_ptr, col_idx, None, blocks, b, spec.m, spec.k, spec.n, rows, nthreads=threads)
    dt = time.perf_counter() - t0
    nblk = int(row_ptr[nrows].item())
    fl = 2.0 * nblk * spec.block * spec.block * spec.n
    desc = (f"block-rows 0..{nrows - 1} of {nbr} ({nblk} of {int(row_ptr[-1].item())} nonzero blocks, "
            f"{fl / 1e9:.1f} GFLOP), fp32-widened inputs, {threads} threads")
    return fl / dt / 1e12, dt, desc, threads


def host_bsr(problem, a):
    """CPU copies of a BSR matrix built on the device and of its dense
    operand as B (K x N); the linear layout's X (N x K) is transposed."""
    b = problem.b.cpu()
    if problem.spec.layout == "linear":
        b = b.t().contiguous()
    blocks = a.blocks.cpu() if a.blk_idx is None else a.blocks[a.blk_idx.long()].cpu()
    return (a.row_ptr.cpu(), a.col_idx.cpu(), blocks, b)


def host_bsr_from_coo(problem):
    """The same BSR matrix built on the host by the reference's convention
    (stable argsort of the tile rows, row offsets from the counts), with the
    oracle: no code of this package's native library is involved."""
    from oracle import oracle

    spec = problem.spec
    perm, _, cols_s = oracle.sort_coo_by_row(problem.mask.indices[0], problem.mask.indices[1], spec.nbr)
    rows_sorted = problem.mask.indices[0].cpu()[perm]
    row_ptr = oracle.row_offsets(rows_sorted, spec.nbr).to(torch.int32)
    tiles = problem.tiles.cpu()
    blocks = tiles if torch.equal(perm, torch.arange(perm.numel())) else tiles[perm].contiguous()
    b = problem.b.cpu()
    if spec.layout == "linear":
        b = b.t().contiguous()
    return (row_ptr, cols_s.to(torch.int32), blocks, b)


# ---------------------------------------------------------------- reference arm

def run_reference(args) -> None:
    """The reference's CPU algorithm for this path on the host cores.  The
    workload is generated with plain torch on the GPU (the same seeded
    inputs as our arm) and copied to the host; the BSR form is built on the
    host by the oracle; the timed work is the oracle alone."""
    rank, world, local = dist_env()
    if rank != 0:
        return
    spec = workload_spec(args)
    if not torch.cuda.is_available():
        raise SystemExit("the reference arm generates its seeded workload on a CUDA device")
    torch.cuda.set_device(local)
    t0 = time.perf_counter()
    problem = generate(spec, seed=args.seed, device="cuda")
    torch.cuda.synchronize()
    host = host_bsr_from_coo(problem)
    log(f"[reference] workload ready in {time.perf_counter() - t0:.1f}s")
    values, secs = [], []
    desc, threads = "", 0
    for i in range(args.warmup + args.steps):
        v, dt, desc, threads = cpu_sample(problem, host, target_s=args.ref_seconds)
        if i >= args.warmup:
            values.append(v)
            secs.append(dt)
    value = statistics.median(values)
    line = {
        "impl": "reference",
        "metric": "bsr_spmm_effective_tflops",
        "value": value,
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": statistics.median(secs) * 1e3,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded)",
        "config": {"workload": spec.name, "m": spec.m, "k": spec.k, "n": spec.n, "block": spec.block,
                   "sparsity": spec.sparsity, "input_dtype": str(spec.dtype).replace("torch.", ""),
                   "parallelism": "cpu"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port", "sample": desc},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- our arm

def run_ours(args) -> None:
    import torch.distributed as dist

    from kairo_b200.ops import KernelConfig, block_sparse_mm_bsr, bsr_from_tiles, describe
    from kairo_b200.sharding import column_range, gather_grid, grid_coords, operand_bytes, partition_rows, shard_bsr

    rank, world, local = dist_env()
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    json_fd = None
    if world > 1:
        from datetime import timedelta

        # The communicator set-up can write a version banner to stdout, where
        # rank 0's one JSON line must stand alone: until that line, file
        # descriptor 1 points at stderr, and the line goes to the saved one.
        sys.stdout.flush()
        json_fd = os.dup(1)
        os.dup2(2, 1)
        if os.environ.get("NCCL_DEBUG", "").upper() in ("", "VERSION"):
            os.environ["NCCL_DEBUG"] = "WARN"
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    spec = workload_spec(args)
    t0 = time.perf_counter()
    problem = generate(spec, seed=args.seed, device=dev)
    a_full = bsr_from_tiles(problem.tiles, problem.row_ids, problem.col_ids, (spec.m, spec.k))
    # Default: the ranks form a (row groups x column slices) grid: within
    # its row group a rank takes an nnz-balanced block-row range, and its
    # column slice is a range of C's (and B's) columns (the batch rows of X
    # in the linear layout); grid_shape picks the shape (2 x 1, 2 x 2, 4 x 2
    # at 2, 4, 8 GPUs for the 262144^2 case).  --rows: block-row ranges
    # only, B replicated.  No collective on the compute path either way.
    row_group, col_slice, row_groups, col_slices = rank, 0, world, 1
    if not args.rows:
        row_group, col_slice, row_groups, col_slices = grid_coords(rank, world, spec.n, 256,
                                                                   *operand_bytes(a_full, spec.n))
    bounds = partition_rows(a_full.row_ptr, row_groups)
    a, shard = shard_bsr(a_full, row_group, row_groups, bounds)
    c0, c1 = column_range(spec.n, col_slices, col_slice)
    ncols = c1 - c0
    local_nnzb = a.nnzb
    local_rows = a.shape[0]
    linear = spec.layout == "linear"
    b = problem.b[c0:c1] if linear else problem.b[:, c0:c1]
    cfg = KernelConfig(kernel=args.kernel, n_tile=args.n_tile, group_blocks=args.group_blocks,
                       schedule=args.schedule, band_rows=args.band_rows, row_cost=args.row_cost,
                       stages=args.stages, num_ctas=args.num_ctas, ctas_per_sm=args.ctas_per_sm,
                       group_rows=args.group_rows)
    t_groups = time.perf_counter()
    plan = describe(a, ncols, linear=linear, config=cfg)  # builds (and caches) row groups when they are used
    groups_build_s = time.perf_counter() - t_groups
    if linear:
        from kairo_b200.ops import sparse_linear

        out = torch.empty(ncols, local_rows, dtype=spec.out_dtype, device=dev)

        def step():
            sparse_linear(b, a, out=out, config=cfg)
    else:
        out = torch.empty(local_rows, ncols, dtype=torch.float32, device=dev)

        def step():
            block_sparse_mm_bsr(a, b, out=out, config=cfg)
    torch.cuda.synchronize()
    log(f"[rank {rank}] workload {spec.name}: grid {row_groups}x{col_slices}, rows {shard.row_begin}..{shard.row_end} "
        f"of {a_full.nbr}, columns {c0}..{c1} of {spec.n}, {local_nnzb} blocks, ready in "
        f"{time.perf_counter() - t0:.1f}s")

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    # Clock samples are taken from the last warm-up steps through the timed
    # region (every 10 ms), so that short timed regions still get samples.
    sampler = ClockSampler(dev)
    with sampler:
        for _ in range(args.warmup):
            flush.zero_()
            step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        wall0 = time.perf_counter()
        for i in range(args.steps):
            flush.zero_()
            starts[i].record(stream)
            step()
            ends[i].record(stream)
        torch.cuda.synchronize()
        wall = time.perf_counter() - wall0
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    per_step = [s.elapsed_time(e) for s, e in zip(starts, ends)]  # ms
    # The device error word of the workspace every timed launch used: a
    # bad index or a timed-out wait in any of them leaves it nonzero.
    from kairo_b200 import _lib

    dev_err = _lib.read_workspace_error(_lib.workspace(0, dev), clear=True)
    l2_peak = l2_gather_peak(flush)
    total_ms = sum(per_step)
    my_ms = total_ms / args.steps
    mine = torch.tensor([my_ms, float(local_nnzb), float(dev_err)], dtype=torch.float64, device=dev)
    if world > 1:
        every = torch.empty(world, 3, dtype=torch.float64, device=dev)
        dist.all_gather_into_tensor(every, mine)
    else:
        every = mine.view(1, 3)
    every = every.cpu()
    rank_ms = every[:, 0].tolist()
    job_ms = max(rank_ms) * args.steps
    ms_per_step = job_ms / args.steps
    dev_errs = sorted({int(x) for x in every[:, 2].tolist()} - {0})
    total_flop = flops(spec)
    value = total_flop / (ms_per_step / 1e3) / 1e12

    peaks, peak_kind = measured_peaks()
    hbm = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    local_spec = dataclasses.replace(spec, n=ncols)
    local_flop = flops(local_spec, nnzb=local_nnzb)
    local_canon = canonical_bytes(local_spec, nnzb=local_nnzb, nbr=a.nbr, m=local_rows)
    local_strict = strict_bytes(local_spec, nnzb=local_nnzb, nbr=a.nbr, m=local_rows)
    traffic = load_traffic(spec.name, world, plan)
    tensor_peak, tensor_peak_kind = compute_peak(spec, plan, peaks, peak_kind)
    roof = strict_roofline(local_flop, local_strict, my_ms, tensor_peak, hbm,
                           "tensor" if plan.get("kernel") in ("tcgen05", "split_bf16") else "fp32")

    # The checker: the whole output of the timed launches against the
    # oracle (outside the timed region).  Each rank checks its own shard.
    parity = None
    if not args.no_check:
        parity = check_output(a, b, out, linear)
        pt = torch.tensor([parity["rel_err"], parity["max_block_row_rel_err"]], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(pt, op=dist.ReduceOp.MAX)
        parity["rel_err"], parity["max_block_row_rel_err"] = pt.tolist()
        parity["scope"] = ("every block-row and column of the output" if world == 1 else
                           "every block-row and column of every rank's shard (max over ranks)")

    # Optional replicated output (reported separately, not part of the step).
    gather_ms = None
    if args.gather and world > 1 and not linear:
        torch.cuda.synchronize()
        dist.barrier()
        g0 = torch.cuda.Event(enable_timing=True)
        g1 = torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        gather_grid(out, bounds, shard.block_rows, spec.m, spec.n, row_groups, col_slices)
        g1.record(stream)
        torch.cuda.synchronize()
        gt = torch.tensor([g0.elapsed_time(g1)], dtype=torch.float64, device=dev)
        dist.all_reduce(gt, op=dist.ReduceOp.MAX)
        gather_ms = gt.item()

    # End to end: host buffers in, the public operator, host result out.
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, spec, a, b, out, cfg, dev, stream, linear, world, dist)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        host = host_bsr(problem, a_full)
        v, dt, desc, threads = cpu_sample(problem, host, target_s=args.cpu_seconds)
        cpu = {"value": v, "unit": "TFLOP/s", "cores": threads, "kind": "port", "sample": desc}

    clocks = sampler.summary()
    if world > 1:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": "bsr_spmm_effective_tflops",
            "value": value,
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_per_step,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": str(spec.dtype).replace("torch.", ""),
            "data": "synthetic (seeded, generated on device)",
            "config": {
                "workload": spec.name, "m": spec.m, "k": spec.k, "n": spec.n, "block": spec.block,
                "sparsity": spec.sparsity, "nnzb": a_full.nnzb, "out_dtype": str(spec.out_dtype).replace("torch.", ""),
                "parallelism": (f"grid {row_groups}x{col_slices} (nnz-balanced block-row groups x column slices "
                                f"of B and C; each column slice of B replicated over the row groups)"),
                "l2": "flushed before every step (256 MiB write, untimed)",
                "kernel_config": {"kernel": args.kernel, "n_tile": args.n_tile, "group_blocks": args.group_blocks,
                                  "row_cost": args.row_cost, "stages": args.stages, "num_ctas": args.num_ctas,
                                  "ctas_per_sm": args.ctas_per_sm,
                                  "schedule": args.schedule, "band_rows": args.band_rows,
                                  "group_rows": args.group_rows, "max_row_blocks": a.max_row_blocks},
                "plan": plan,
                **({"row_groups_build_ms": round(groups_build_s * 1e3, 3)} if plan["schedule"] == "groups" else {}),
            },
            "roofline": {
                **roof,
                "traffic": traffic,
                "peak_kind": peak_kind if roof["bound"] == "hbm" else tensor_peak_kind,
                "definition": ("max(FLOP / tensor peak, strict bytes / HBM bandwidth) for rank 0's shard, over "
                               "its mean kernel time; strict bytes = A blocks + int32 indices + B once + C"),
                "traffic_source": ("ncu capture of this launch plan (profiles/traffic_<workload>.txt)"
                                   if traffic is not None else "no capture of this launch plan"),
                # canonical bytes count one gathered B panel per block; most
                # of those come from L2, so this fraction can exceed 1
                "canonical_gbs": local_canon / (my_ms / 1e3) / 1e9,
                "canonical_frac": local_canon / (my_ms / 1e3) / 1e9 / hbm,
                # the same canonical bytes against this GPU's measured L2 -> SM
                # bulk-copy ceiling (kairo_gather_probe), measured live
                "l2_gather_peak_gbs": l2_peak,
                "l2_frac": (local_canon / (my_ms / 1e3) / 1e9 / l2_peak) if l2_peak else None,
            },
            "parity": parity,
            "parity_rel_err": None if parity is None else parity["rel_err"],
            "device_errors": dev_errs,
            "ranks": {"kernel_ms_min": min(rank_ms), "kernel_ms_median": statistics.median(rank_ms),
                      "kernel_ms_max": max(rank_ms), "nnzb_min": int(every[:, 1].min()),
                      "nnzb_max": int(every[:, 1].max())},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": args.steps * plan["launches"],
            "clocks": clocks,
            "wall_s_timed_region": wall,
        }
        if gather_ms is not None:
            line["gather_ms"] = gather_ms
        if json_fd is not None:
            sys.stdout.flush()
            os.write(json_fd, (json.dumps(line) + "\n").encode())
        else:
            print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_e2e(args, spec, a, b, out, cfg, dev, stream, linear, world, dist):
    """Same metric through the public operator with host (pinned) buffers:
    every step copies this rank's blocks, indices and B to the device and
    reads C back; the copies are inside the timed region.  Consecutive steps
    are pipelined the way a serving loop overlaps requests: two device buffer
    sets and three streams (upload, compute, read-back), so step i's read-back
    runs while step i+1 uploads (PCIe is full duplex).  A set is reused only
    after its previous read-back has finished."""
    from kairo_b200.ops import block_sparse_mm_bsr, sparse_linear
    from kairo_b200.types import BlockSparseMatrix

    b = b.contiguous()  # this rank's columns of B (rows of X) as one host buffer
    h_blocks = a.blocks.to("cpu").pin_memory()
    h_rp = a.row_ptr.to("cpu").pin_memory()
    h_ci = a.col_idx.to("cpu").pin_memory()
    h_b = b.to("cpu").pin_memory()
    h_out = [torch.empty(out.shape, dtype=out.dtype).pin_memory() for _ in range(2)]
    sets = [{"blocks": torch.empty_like(a.blocks), "rp": torch.empty_like(a.row_ptr),
             "ci": torch.empty_like(a.col_idx), "b": torch.empty_like(b),
             "out": out if j == 0 else torch.empty_like(out)} for j in range(2)]
    s_in = torch.cuda.Stream(dev)
    s_out = torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_c = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    used = [False, False]
    steps = max(1, min(args.steps, args.e2e_steps))

    def one(i):
        j = i % 2
        d = sets[j]
        with torch.cuda.stream(s_in):
            if used[j]:
                s_in.wait_event(ev_out[j])   # set j's last read-back (and so its compute) is done
            d["blocks"].copy_(h_blocks, non_blocking=True)
            d["rp"].copy_(h_rp, non_blocking=True)
            d["ci"].copy_(h_ci, non_blocking=True)
            d["b"].copy_(h_b, non_blocking=True)
            ev_in[j].record(s_in)
        used[j] = True
        stream.wait_event(ev_in[j])
        m = BlockSparseMatrix(row_ptr=d["rp"], col_idx=d["ci"], blocks=d["blocks"], shape=a.shape,
                              block_size=a.block_size, max_row_blocks=a.max_row_blocks)
        if linear:
            sparse_linear(d["b"], m, out=d["out"], config=cfg)
        else:
            block_sparse_mm_bsr(m, d["b"], out=d["out"], config=cfg)
        ev_c[j].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_c[j])
            h_out[j].copy_(d["out"], non_blocking=True)
            ev_out[j].record(s_out)
        return j

    for i in range(2):  # warm-up of both sets
        one(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(s_in)
    last = 0
    for i in range(steps):
        last = one(i)
    stream.wait_event(ev_out[last])
    stream.wait_event(ev_out[1 - last])
    e1.record(stream)
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = t.item()
    h2d = h_blocks.numel() * h_blocks.element_size() + h_rp.numel() * 4 + h_ci.numel() * 4 + h_b.numel() * h_b.element_size()
    d2h = h_out[0].numel() * h_out[0].element_size()
    if world > 1:
        tb = torch.tensor([float(h2d), float(d2h)], dtype=torch.float64, device=dev)
        dist.all_reduce(tb, op=dist.ReduceOp.SUM)
        h2d, d2h = int(tb[0].item()), int(tb[1].item())
    return {"value": flops(spec) / (ms / 1e3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms,
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "steps": steps,
            "path": "pinned host -> device copies, kairo_b200.ops.block_sparse_mm_bsr, device -> pinned host; "
                    "consecutive steps overlapped on upload / compute / read-back streams"}


# ---------------------------------------------------------------- backward

def run_backward(args) -> None:
    """One training-step backward of the linear layer Y = X @ W^T with the
    linear-layer workload's weight: refresh W^T's values, dX = dY @ W (the
    LINEAR SpMM on W^T) and dW on W's nonzero blocks (SDDMM, bf16 output).
    Each part is timed with its own CUDA events; the step is their sum."""
    from kairo_b200.ops import (KernelConfig, bsr_from_tiles, bsr_transpose, describe, sparse_linear,
                                sparse_linear_weight_grad, transpose_values)

    rank, world, local = dist_env()
    if world > 1:
        raise SystemExit("--op backward runs on one GPU")
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    spec = WORKLOADS[args.workload if args.workload != "bf16_uniform" else "bf16_linear"]
    if args.shape:
        m, k, n = (int(x) for x in args.shape.lower().split("x"))
        spec = spec.scaled(m, k, n)
    if spec.layout != "linear":
        raise SystemExit("--op backward needs a linear-layout workload (bf16_linear)")
    problem = generate(spec, seed=args.seed, device=dev)
    w = bsr_from_tiles(problem.tiles, problem.row_ids, problem.col_ids, (spec.m, spec.k))
    x = problem.b                                     # (batch, in_features)
    g = torch.Generator(device=dev).manual_seed(args.seed + 1)
    dy = torch.randn(spec.n, spec.m, generator=g, device=dev).to(spec.dtype)
    wt = bsr_transpose(w, check=True)
    dx = torch.empty(spec.n, spec.k, dtype=spec.dtype, device=dev)
    cfg = KernelConfig(n_tile=args.n_tile, group_blocks=args.group_blocks, schedule=args.schedule,
                       band_rows=args.band_rows, ctas_per_sm=args.ctas_per_sm)
    parts = ("wt_values", "dx", "dw")

    def part(name):
        if name == "wt_values":
            transpose_values(w, wt)
        elif name == "dx":
            sparse_linear(dy, wt.matrix, out=dx, config=cfg)
        else:
            sparse_linear_weight_grad(dy, x, w, wt, out_dtype=spec.dtype)

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    times = {p: [] for p in parts}
    sampler = ClockSampler(dev)
    with sampler:
        for i in range(args.warmup + args.steps):
            for p in parts:
                flush.zero_()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                part(p)
                e1.record(stream)
                if i >= args.warmup:
                    times[p].append((e0, e1))
        torch.cuda.synchronize()
    ms = {p: sum(a.elapsed_time(b) for a, b in times[p]) / args.steps for p in parts}
    step_ms = sum(ms.values())
    fl = flops(spec)  # one product: 2 * nnzb * bm * bk * batch
    peaks, peak_kind = measured_peaks()
    tpeak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    sdd_tflops = fl / (ms["dw"] / 1e3) / 1e12
    line = {
        "metric": "linear_backward_tflops",
        "value": 2 * fl / (step_ms / 1e3) / 1e12,
        "unit": "TFLOP/s",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": step_ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": str(spec.dtype).replace("torch.", ""),
        "data": "synthetic (seeded, generated on device)",
        "config": {"workload": spec.name, "m": spec.m, "k": spec.k, "batch": spec.n, "block": spec.block,
                   "sparsity": spec.sparsity, "nnzb": w.nnzb, "parts_ms": ms,
                   "dx_plan": describe(wt.matrix, spec.n, linear=True, config=cfg),
                   "l2": "flushed before every part (256 MiB write, untimed)"},
        "roofline": {"bound": "tensor", "kernel": "bsr_sddmm_tc (dW)", "achieved": sdd_tflops, "peak": tpeak,
                     "unit": "TFLOP/s", "frac": sdd_tflops / tpeak, "traffic": None, "peak_kind": peak_kind},
        "cpu_baseline": None,
        # values refresh 1, dX per its plan, dW: stack list + SDDMM 2
        "gpu_launches": args.steps * (1 + describe(wt.matrix, spec.n, linear=True, config=cfg)["launches"] + 2),
        "clocks": sampler.summary(),
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- autotuner

def run_tune(args) -> None:
    """The autotuner's candidates on a named workload: every launch variant
    of BLACKWELL_VARIANTS and GROUP_VARIANTS (the first is the library
    default) timed on the actual
    matrix by TileAutotuner.time_kernel_configs (CUDA events, median of
    BENCH_ITERS, L2 not flushed between calls), and the one
    best_kernel_config picks.  Evidence for the library's defaults."""
    from kairo_b200.ops import TileAutotuner, bsr_from_tiles, describe

    rank, world, local = dist_env()
    if world > 1:
        raise SystemExit("--op tune runs on one GPU")
    torch.cuda.set_device(local)
    spec = workload_spec(args)
    if spec.layout == "linear":
        raise SystemExit("--op tune times the STANDARD layout; the linear layer's X^T is its B")
    problem = generate(spec, seed=args.seed, device="cuda")
    a = bsr_from_tiles(problem.tiles, problem.row_ids, problem.col_ids, (spec.m, spec.k))
    tuner = TileAutotuner()
    rows = []
    for kc, ms in tuner.time_kernel_configs(a, spec.n, B=problem.b):
        try:
            plan = describe(a, spec.n, config=kc)
        except Exception as exc:  # noqa: BLE001 - a variant this shape does not support
            plan = {"unsupported": str(exc)}
        rows.append({"n_tile": kc.n_tile, "stages": kc.stages, "row_cost": kc.row_cost, "schedule": kc.schedule,
                     "group_blocks": kc.group_blocks, "ctas_per_sm": kc.ctas_per_sm, "group_rows": kc.group_rows,
                     "ms": ms,
                     "tflops": flops(spec) / (ms / 1e3) / 1e12,
                     "plan": plan})
    best = tuner.best_kernel_config(a, spec.n)
    print(json.dumps({"op": "tune", "workload": spec.name, "candidates": rows,
                      "best": dataclasses.asdict(best), "default_plan": describe(a, spec.n)}), flush=True)


# ---------------------------------------------------------------- block pruning

def run_prune(args) -> None:
    """The linear layer's mask generator as a step: block L2 norms of the
    dense weight (8192 x 32768 bf16, 64 x 64 blocks) and the top 20 % of the
    65536 block scores, indices ascending (block_magnitude_mask).  HBM-bound:
    the weight is read once."""
    from kairo_b200.pruning import block_magnitude_mask, block_norms, topk_indices

    rank, world, local = dist_env()
    if world > 1:
        raise SystemExit("--op prune runs on one GPU")
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    m, k, bs, keep = 8192, 32768, 64, 0.2
    g = torch.Generator(device=dev).manual_seed(args.seed)
    w = (torch.randn(m, k, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    nblocks = (m // bs) * (k // bs)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    ev = []
    sampler = ClockSampler(dev)
    with sampler:
        for i in range(args.warmup + args.steps):
            flush.zero_()
            e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
            e0.record(stream)
            scores = block_norms(w, bs)
            e1.record(stream)
            idx = topk_indices(scores, int(nblocks * keep))
            e2.record(stream)
            if i >= args.warmup:
                ev.append((e0, e1, e2))
        torch.cuda.synchronize()
    norms_ms = sum(a.elapsed_time(b) for a, b, _ in ev) / args.steps
    topk_ms = sum(b.elapsed_time(c) for _, b, c in ev) / args.steps
    ms = norms_ms + topk_ms
    mask = block_magnitude_mask(w, bs, keep)  # the public call, checked against the two parts
    assert torch.equal(mask.indices[0] * (k // bs) + mask.indices[1], idx)
    nbytes = m * k * 2 + nblocks * 4
    peaks, peak_kind = measured_peaks()
    hbm = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    achieved = nbytes / (norms_ms / 1e3) / 1e9

    cpu = None
    if not args.no_cpu:
        # The reference's rule with torch on the host (per-block norm, topk,
        # sort) on the first 512 block-columns' worth of rows: 1/16 of W.
        hw = w[: m // 16].float().cpu()
        t0 = time.perf_counter()
        sc = hw.view(m // 16 // bs, bs, k // bs, bs).pow(2).sum(dim=(1, 3)).sqrt()
        torch.topk(sc.reshape(-1), int(sc.numel() * keep)).indices.sort()
        dt = time.perf_counter() - t0
        cpu = {"value": (m // 16) * k * 2 / dt / 1e9, "unit": "GB/s", "cores": torch.get_num_threads(),
               "kind": "port", "sample": f"rows 0..{m // 16 - 1} of the weight (1/16), torch on the host"}
    line = {
        "metric": "block_prune_weight_gbs",
        "value": m * k * 2 / (ms / 1e3) / 1e9,
        "unit": "GB/s",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded, generated on device)",
        "config": {"workload": "linear-layer mask: top 20 % of 64x64 blocks of 8192x32768 bf16", "m": m, "k": k,
                   "block": bs, "keep": keep, "parts_ms": {"block_norms": norms_ms, "topk": topk_ms},
                   "l2": "flushed before every step (256 MiB write, untimed)"},
        "roofline": {"bound": "hbm", "kernel": "block norms", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "traffic": None, "peak_kind": peak_kind},
        "cpu_baseline": cpu,
        "gpu_launches": args.steps * 13,  # block norms 1; top-k: init, 4 x (histogram, pick), count, scan, write
        "clocks": sampler.summary(),
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- embedding ops

EMB_WORKLOADS = {
    # the reference's embedding benchmark shape (benchmarks/bench_embedding.py:
    # 35-46: 10000 x 64 table, batch 256, 80 % sparse mask), fp32
    "emb_ref_bench": {"n": 10000, "d": 64, "batch": 256, "sparsity": 0.8},
    # a production-sized table: 1M x 128 fp32 (512 MiB), batch 65536
    "emb_large": {"n": 1_000_000, "d": 128, "batch": 65536, "sparsity": 0.8},
}


def emb_problem(name: str, dev, seed: int):
    """Seeded table, element mask (each entry active with probability
    1 - sparsity, row-major order) and a batch of uniform ids with repeats."""
    from kairo_b200.types import SparseMask

    w = EMB_WORKLOADS[name]
    g = torch.Generator(device=dev).manual_seed(seed)
    n, d, b = w["n"], w["d"], w["batch"]
    weight = torch.randn(n, d, generator=g, device=dev)
    keep = torch.rand(n, d, generator=g, device=dev) >= w["sparsity"]
    idx = keep.nonzero().t().contiguous()
    del keep
    mask = SparseMask(indices=idx, values=torch.ones(idx.shape[1], device=dev), dense_shape=(n, d),
                      sparsity_ratio=w["sparsity"])
    ids = torch.randint(0, n, (b,), generator=g, device=dev)
    grad = torch.randn(b, d, generator=g, device=dev)
    return w, weight, mask, ids, grad


def emb_bytes(op: str, w: dict, ids, active) -> float:
    """Algorithmic bytes of one launch (fp32): gather reads every id, its
    row's mask bits (D / 8 bytes) and weight row, and writes the output row;
    scatter writes the dense gradient once and reads the batch ids, the
    gradient rows and the active ids."""
    d, b = w["d"], w["batch"]
    if op == "gather":
        return float(b * (8 + (d + 31) // 32 * 4 + 2 * 4 * d))
    return float(w["n"] * d * 4 + b * (8 + 4 * d) + active.numel() * 8)


def run_embedding(args) -> None:
    from kairo_b200.ops import sort_mask_rows, sparse_gather, sparse_scatter_grad

    rank, world, local = dist_env()
    if world > 1:
        raise SystemExit("--op gather/scatter runs on one GPU (independent replicas need no collective)")
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    name = args.emb_workload
    w, weight, mask, ids, grad = emb_problem(name, dev, args.seed)
    mr = sort_mask_rows(mask)
    active = torch.unique(ids)
    n, d = w["n"], w["d"]
    out = None

    if args.op == "gather":
        def step():
            return sparse_gather(weight, mr, ids)
    else:
        def step():
            return sparse_scatter_grad(grad, active, ids, n, d)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    sampler = ClockSampler(dev)
    with sampler:
        for _ in range(args.warmup):
            flush.zero_()
            out = step()
        torch.cuda.synchronize()
        for i in range(args.steps):
            flush.zero_()
            starts[i].record(stream)
            out = step()
            ends[i].record(stream)
        torch.cuda.synchronize()
    ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / args.steps
    rows_per_s = w["batch"] / (ms / 1e3)
    # Reference point: a device-to-device copy of the result's bytes, timed
    # the same way (flush, events), shows what a transfer of this size reaches.
    src = weight.reshape(-1)[: out.numel()]
    dst = torch.empty_like(src)
    copy_ms = []
    for i in range(args.warmup + args.steps):
        flush.zero_()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(stream)
        dst.copy_(src)
        c1.record(stream)
        torch.cuda.synchronize()
        if i >= args.warmup:
            copy_ms.append(c0.elapsed_time(c1))
    copy_gbs = 2 * src.numel() * 4 / (statistics.median(copy_ms) / 1e3) / 1e9
    del dst
    nbytes = emb_bytes(args.op, w, ids, active)
    peaks, peak_kind = measured_peaks()
    hbm = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    achieved = nbytes / (ms / 1e3) / 1e9

    # End to end: ids (and the gradient rows) from pinned host memory, the
    # result back to pinned host memory, inside the timed region.
    h_ids = ids.cpu().pin_memory()
    h_grad = grad.cpu().pin_memory() if args.op == "scatter" else None
    h_active = active.cpu().pin_memory()
    h_out = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    d_ids = torch.empty_like(ids)
    d_grad = torch.empty_like(grad) if args.op == "scatter" else None
    d_active = torch.empty_like(active)

    def one():
        d_ids.copy_(h_ids, non_blocking=True)
        if args.op == "gather":
            r = sparse_gather(weight, mr, d_ids)
        else:
            d_grad.copy_(h_grad, non_blocking=True)
            d_active.copy_(h_active, non_blocking=True)
            r = sparse_scatter_grad(d_grad, d_active, d_ids, n, d)
        h_out.copy_(r, non_blocking=True)

    one()
    torch.cuda.synchronize()
    e_steps = max(1, min(args.steps, args.e2e_steps))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e_steps):
        one()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e_steps
    h2d = h_ids.numel() * 8 + (h_grad.numel() * 4 + h_active.numel() * 8 if args.op == "scatter" else 0)
    d2h = h_out.numel() * h_out.element_size()

    cpu = None
    if not args.no_cpu:
        cpu = emb_cpu_sample(args.op, w, weight, mr, ids, grad, active, args.cpu_seconds)
    line = {
        "metric": f"embedding_{args.op}_rows_per_s",
        "value": rows_per_s,
        "unit": "rows/s",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded, generated on device)",
        "config": {"workload": name, **w, "mask_nnz": mr.nnz, "active_rows": int(active.numel()),
                   "parallelism": "single GPU", "l2": "flushed before every step (256 MiB write, untimed)"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "traffic": None, "peak_kind": peak_kind,
                     "copy_same_size_gbs": copy_gbs,
                     "bytes_definition": ("ids + row mask bits + weight rows + output rows"
                                          if args.op == "gather" else
                                          "dense gradient write + batch ids + gradient rows + active ids")},
        "cpu_baseline": cpu,
        "e2e": {"value": w["batch"] / (e2e_ms / 1e3), "unit": "rows/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "steps": e_steps},
        # scatter: keys, count, scan (one CTA, or three kernels above 16384
        # buckets), place, segment sort, sums
        "gpu_launches": args.steps * (1 if args.op == "gather" else (6 if active.numel() + 1 <= 16384 else 8)),
        "clocks": sampler.summary(),
    }
    print(json.dumps(line), flush=True)


def emb_cpu_sample(op, w, weight, mr, ids, grad, active, target_s: float):
    """The oracle (one thread) on the first ids of the batch, sized for about
    ``target_s`` seconds; rows/s."""
    from oracle import oracle

    ro = mr.row_offsets.cpu()
    cols = mr.cols.cpu()
    h_ids = ids.cpu()
    if op == "gather":
        hw = weight.cpu()
        t0 = time.perf_counter()
        oracle.sparse_gather(hw, ro, cols, h_ids)
        dt = time.perf_counter() - t0
        desc = f"all {h_ids.numel()} ids of the batch, 1 thread"
        return {"value": h_ids.numel() / dt, "unit": "rows/s", "cores": 1, "kind": "port", "sample": desc}
    hg = grad.cpu()
    ha = active.cpu()
    t0 = time.perf_counter()
    oracle.sparse_scatter_grad(hg, ha, h_ids, w["n"], w["d"])
    dt = time.perf_counter() - t0
    desc = f"the whole batch ({h_ids.numel()} rows) into the {w['n']} x {w['d']} gradient, 1 thread"
    return {"value": h_ids.numel() / dt, "unit": "rows/s", "cores": 1, "kind": "port", "sample": desc}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="bf16_uniform")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--shape", default="", help="MxKxN override of the workload's sizes (same density), "
                    "for profiling smaller cases")
    ap.add_argument("--sparsity", type=float, default=None, help="block sparsity override of the workload")
    ap.add_argument("--kernel", choices=("auto", "simt", "tcgen05", "split_bf16"), default="auto",
                    help="kernel family (split_bf16: fp32 workloads on the tensor cores, opt-in)")
    ap.add_argument("--n-tile", type=int, default=0)
    ap.add_argument("--group-blocks", type=int, default=0)
    ap.add_argument("--schedule", choices=("auto", "rows", "bands", "groups"), default="auto")
    ap.add_argument("--group-rows", type=int, default=0, help="block-rows per row group (2, 4, 8; 0 = 4)")
    ap.add_argument("--band-rows", type=int, default=0)
    ap.add_argument("--row-cost", type=int, default=0, help="scheduler weight of a block-row (0 = library default)")
    ap.add_argument("--stages", type=int, default=0, help="pipeline stages of the tcgen05 kernel (0 = library default)")
    ap.add_argument("--num-ctas", type=int, default=0, help="persistent grid size (0 = library default)")
    ap.add_argument("--ctas-per-sm", type=int, default=0, help="resident CTAs per SM (0 = library default)")
    ap.add_argument("--gather", action="store_true", help="also time the all-gather of C (reported separately)")
    ap.add_argument("--rows", action="store_true",
                    help="at N > 1 split A into nnz-balanced block-row ranges only, B replicated "
                         "(default: a grid of block-row groups x column slices of B and C)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=8)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-check", action="store_true",
                    help="skip the check of the timed launches' output against the oracle")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ref-seconds", type=float, default=3.0)
    ap.add_argument("--op", choices=("spmm", "backward", "prune", "gather", "scatter", "tune"), default="spmm",
                    help="spmm (default): the block-sparse SpMM; backward: the linear layer's dX and dW; "
                         "prune: block norms + top-k of the linear layer's weight; "
                         "gather/scatter: the masked embedding ops")
    ap.add_argument("--emb-workload", choices=sorted(EMB_WORKLOADS), default="emb_large")
    args = ap.parse_args()
    if args.warmup < 3:
        log("warning: fewer than 3 warm-up steps")
    if args.op != "spmm":
        if args.impl == "reference":
            raise SystemExit("--impl reference times the SpMM path only")
        if args.op == "backward":
            run_backward(args)
        elif args.op == "tune":
            run_tune(args)
        elif args.op == "prune":
            run_prune(args)
        else:
            run_embedding(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
