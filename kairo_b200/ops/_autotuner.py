"""Runtime tile / launch-shape selection for the block-sparse SpMM.

Keeps the reference's entry point and contract (kairo/ops/_autotuner.py:15-191):
``TileConfig``, ``CANDIDATE_CONFIGS``, ``DEFAULT_CONFIG``, ``BENCH_WARMUP``,
``BENCH_ITERS``, ``_cache_key``, and ``TileAutotuner.best_config(M, K, N,
sparsity)`` returning a dict with ``tile_m``, ``tile_n`` and ``tile_k``,
cached in ``TileAutotuner._cache`` and cleared by ``clear_cache()``.

On B200 the search space gains the Blackwell launch knobs of the tcgen05
kernel (``BLACKWELL_VARIANTS``): ``n_tile`` (128 or 256 columns of C per work
item, i.e. one or two M=128 MMAs sharing each block), ``stages``
(shared-memory pipeline depth), ``row_cost`` (scheduler weight of a
block-row), ``schedule`` (row split, bands or row groups of
``GROUP_VARIANTS`` rows), ``group_blocks`` (blocks
per pipeline stage) and ``ctas_per_sm`` (resident CTAs per SM).  They are returned as extra keys.  Candidate tiles are
built as tile_m x tile_k blocks (the reference times square tile_m tiles
whatever tile_k is), so each candidate is timed with the kernel it would
get.  Timing uses CUDA events (median of ``BENCH_ITERS``) instead of host
wall-clock.  ``best_config`` can be told the input dtype and, when the
caller's mask has a fixed block size, that block size; both enter the cache
key.  Without CUDA, ``best_config`` returns ``DEFAULT_CONFIG`` like the
reference.
"""

from __future__ import annotations

import logging
from dataclasses import dataclass
from typing import Any

import torch

_logger = logging.getLogger(__name__)


@dataclass(frozen=True)
class TileConfig:
    """Immutable tile configuration for block-sparse matmul.

    tile_m/tile_n/tile_k: the reference's keys; tile_m x tile_k is the block
    shape of the timing run.  n_tile, stages, row_cost, schedule,
    group_blocks: tcgen05 launch knobs (0 / "auto" = library default).
    """

    tile_m: int
    tile_n: int
    tile_k: int
    n_tile: int = 0
    stages: int = 0
    row_cost: int = 0
    schedule: str = "auto"
    group_blocks: int = 0
    ctas_per_sm: int = 0

    def __post_init__(self) -> None:
        if min(self.tile_m, self.tile_n, self.tile_k) <= 0:
            raise ValueError("tile sizes must be positive")
        if self.n_tile not in (0, 128, 256):
            raise ValueError("n_tile must be 0, 128 or 256")
        if self.stages < 0 or self.row_cost < 0 or self.group_blocks < 0 or self.ctas_per_sm < 0:
            raise ValueError("stages, row_cost, group_blocks and ctas_per_sm must be non-negative")
        if self.schedule not in ("auto", "rows", "bands"):
            raise ValueError("schedule must be 'auto', 'rows' or 'bands'")

    def kernel_config(self):
        from kairo_b200.ops.spmm import KernelConfig

        return KernelConfig(n_tile=self.n_tile, stages=self.stages, row_cost=self.row_cost,
                            schedule=self.schedule, group_blocks=self.group_blocks, ctas_per_sm=self.ctas_per_sm)


# Reference candidates (_autotuner.py:25-31), kept for the legacy keys.
CANDIDATE_CONFIGS: tuple[TileConfig, ...] = (
    TileConfig(tile_m=16, tile_n=16, tile_k=16),
    TileConfig(tile_m=32, tile_n=32, tile_k=16),
    TileConfig(tile_m=64, tile_n=64, tile_k=16),
    TileConfig(tile_m=16, tile_n=16, tile_k=32),
    TileConfig(tile_m=32, tile_n=32, tile_k=32),
)

DEFAULT_CONFIG = CANDIDATE_CONFIGS[0]

# Blackwell launch variants tried for 16-bit inputs on top of each tile size:
# (n_tile, stages, row_cost, schedule, group_blocks, ctas_per_sm).
BLACKWELL_VARIANTS: tuple[tuple[int, int, int, str, int, int], ...] = (
    (0, 0, 0, "auto", 0, 0),
    (128, 0, 0, "auto", 0, 0),
    (256, 0, 0, "auto", 0, 0),
    (0, 0, 0, "rows", 0, 1),
    (0, 0, 0, "rows", 0, 2),
    (0, 0, 0, "bands", 0, 0),
    (0, 0, 0, "bands", 0, 1),
    (128, 0, 4, "rows", 0, 0),
    (0, 0, 0, "rows", 2, 2),
    (0, 0, 0, "rows", 8, 1),
    (256, 4, 0, "rows", 0, 1),
)

# Row-group sizes also timed by ``time_kernel_configs`` (schedule "groups";
# a matrix the row groups do not support times as inf).
GROUP_VARIANTS: tuple[int, ...] = (2, 4)

BENCH_WARMUP = 2
BENCH_ITERS = 5


def _cache_key(M: int, K: int, N: int, sparsity: float, dtype: torch.dtype | None = None,
               block: int | None = None) -> str:
    """Bucketed key (dims to {128, 512, 2048, 4096}, sparsity to 0.1), as the
    reference's; plus the dtype (16-bit inputs run other kernels than fp32)
    and, when the caller fixes it, the block size."""

    def bucket(x: int) -> int:
        if x <= 128:
            return 128
        if x <= 512:
            return 512
        if x <= 2048:
            return 2048
        return 4096

    sp_bucket = round(sparsity, 1)
    key = f"{bucket(M)}_{bucket(K)}_{bucket(N)}_{sp_bucket}"
    if dtype is not None and dtype != torch.float32:
        key += f"_{str(dtype).replace('torch.', '')}"
    if block is not None:
        key += f"_b{int(block)}"
    return key


class TileAutotuner:
    """Benchmarks candidate configurations and caches the best per key."""

    def __init__(self) -> None:
        self._cache: dict[str, dict[str, Any]] = {}

    def best_config(
        self,
        M: int,
        K: int,
        N: int,
        sparsity: float,
        dtype: torch.dtype = torch.float32,
        block: int | None = None,
    ) -> dict[str, Any]:
        """Best configuration for the problem size.

        Returns a dict with 'tile_m', 'tile_n', 'tile_k' (and the Blackwell
        keys 'n_tile', 'stages', 'row_cost', 'schedule', 'group_blocks').
        ``block`` restricts the search to square tiles of that size (a mask
        of fixed granularity).  Without CUDA, or if every candidate fails,
        the default config is returned.
        """
        key = _cache_key(M, K, N, sparsity, dtype, block)
        if key in self._cache:
            return self._cache[key]
        if not torch.cuda.is_available():
            result = _config_to_dict(DEFAULT_CONFIG if block is None else TileConfig(block, block, block))
            self._cache[key] = result
            return result
        best = self._benchmark(M, K, N, sparsity, dtype, block)
        self._cache[key] = best
        return best

    def candidates(self, M: int, K: int, dtype: torch.dtype, block: int | None = None) -> list[TileConfig]:
        """Every (tile, launch variant) pair ``best_config`` times."""
        tiles = CANDIDATE_CONFIGS if block is None else (TileConfig(block, block, block),)
        out = []
        for cfg in tiles:
            if cfg.tile_m > M or cfg.tile_k > K:
                continue
            square16 = dtype in (torch.float16, torch.bfloat16) and cfg.tile_m == cfg.tile_k
            variants = BLACKWELL_VARIANTS if square16 else ((0, 0, 0, "auto", 0, 0),)
            for n_tile, stages, row_cost, schedule, group, per_sm in variants:
                out.append(TileConfig(cfg.tile_m, cfg.tile_n, cfg.tile_k, n_tile, stages, row_cost, schedule, group,
                                      per_sm))
        return out

    def _benchmark(self, M: int, K: int, N: int, sparsity: float, dtype: torch.dtype,
                   block: int | None = None) -> dict[str, Any]:
        best_time = float("inf")
        best_cfg = DEFAULT_CONFIG if block is None else TileConfig(block, block, block)
        for cand in self.candidates(M, K, dtype, block):
            elapsed = self._time_config(cand, M, K, N, sparsity, dtype)
            if elapsed < best_time:
                best_time = elapsed
                best_cfg = cand
        return _config_to_dict(best_cfg)

    def _time_config(self, cfg: TileConfig, M: int, K: int, N: int, sparsity: float,
                     dtype: torch.dtype = torch.float32) -> float:
        """Median time in seconds of one BSR SpMM with ``cfg`` on random data
        at the given sparsity: a random mask of tile_m x tile_k blocks."""
        try:
            from kairo_b200.ops.spmm import block_sparse_mm_bsr, bsr_from_tiles

            device = torch.device("cuda")
            bm, bk = cfg.tile_m, cfg.tile_k
            nbr = (M + bm - 1) // bm
            nbc = (K + bk - 1) // bk
            total = nbr * nbc
            nnz = max(1, int(total * (1.0 - sparsity)))
            perm = torch.randperm(total, device=device)[:nnz]
            rows = (perm // nbc).to(torch.int32)
            cols = (perm % nbc).to(torch.int32)
            tiles = torch.randn(nnz, bm, bk, device=device).to(dtype)
            B = torch.randn(K, N, device=device).to(dtype)
            a = bsr_from_tiles(tiles, rows, cols, (M, K))
            out = torch.empty(M, N, dtype=torch.float32, device=device)
            kc = cfg.kernel_config()
            return _median_seconds(lambda: block_sparse_mm_bsr(a, B, out=out, config=kc))
        except Exception as exc:  # noqa: BLE001 - a failing candidate is skipped, as in the reference
            _logger.debug("Autotuner config %s failed: %s", cfg, exc)
            return float("inf")

    def time_kernel_configs(self, a, N: int, candidates=None, B=None) -> list[tuple[Any, float]]:  # noqa: ANN001
        """(KernelConfig, median ms) of every candidate on an actual
        BlockSparseMatrix ``a`` with N columns (CUDA events); a candidate
        that fails gets inf.  ``B`` defaults to random data of a's dtype."""
        from kairo_b200.ops.spmm import KernelConfig, block_sparse_mm_bsr

        if candidates is None:
            candidates = [KernelConfig(n_tile=nt, stages=st, row_cost=rc, schedule=sc, group_blocks=gb,
                                       ctas_per_sm=per_sm)
                          for nt, st, rc, sc, gb, per_sm in BLACKWELL_VARIANTS]
            candidates += [KernelConfig(schedule="groups", group_rows=rg) for rg in GROUP_VARIANTS]
        if B is None:
            B = torch.randn(a.shape[1], N, device=a.device).to(a.dtype)
        out = torch.empty(a.shape[0], N, dtype=torch.float32, device=a.device)
        result = []
        for kc in candidates:
            try:
                ms = _median_seconds(lambda: block_sparse_mm_bsr(a, B, out=out, config=kc)) * 1e3
            except Exception as exc:  # noqa: BLE001
                _logger.debug("kernel config %s failed: %s", kc, exc)
                ms = float("inf")
            result.append((kc, ms))
        return result

    def best_kernel_config(self, a, N: int, candidates=None):  # noqa: ANN001
        """Best :class:`KernelConfig` for an actual BlockSparseMatrix ``a``
        and N columns, timed on that matrix (CUDA events, median)."""
        from kairo_b200.ops.spmm import KernelConfig

        key = f"bsr_{a.shape}_{a.block_size}_{a.nnzb}_{a.max_row_blocks}_{N}_{a.dtype}"
        if key in self._cache:
            return KernelConfig(**self._cache[key])
        timed = self.time_kernel_configs(a, N, candidates)
        best, best_t = KernelConfig(), float("inf")
        for kc, t in timed:
            if t < best_t:
                best, best_t = kc, t
        self._cache[key] = {"kernel": best.kernel, "n_tile": best.n_tile, "stages": best.stages,
                            "row_cost": best.row_cost, "num_ctas": best.num_ctas, "schedule": best.schedule,
                            "group_blocks": best.group_blocks, "band_rows": best.band_rows,
                            "ctas_per_sm": best.ctas_per_sm, "group_rows": best.group_rows}
        return best

    def clear_cache(self) -> None:
        """Clear the autotuner cache."""
        self._cache.clear()


def _median_seconds(run) -> float:  # noqa: ANN001
    """Median of BENCH_ITERS CUDA-event timings of ``run`` after
    BENCH_WARMUP calls.  Before each start event the stream is kept busy for
    about 50 us, so that the host's own work of the call (argument checks,
    the ctypes call) overlaps device work and the events time the kernels,
    not the host."""
    for _ in range(BENCH_WARMUP):
        run()
    torch.cuda.synchronize()
    times: list[float] = []
    for _ in range(BENCH_ITERS):
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(100_000)
        start.record()
        run()
        end.record()
        end.synchronize()
        times.append(start.elapsed_time(end) / 1e3)
    times.sort()
    return times[len(times) // 2]


def _config_to_dict(cfg: TileConfig) -> dict[str, Any]:
    return {
        "tile_m": cfg.tile_m,
        "tile_n": cfg.tile_n,
        "tile_k": cfg.tile_k,
        "n_tile": cfg.n_tile,
        "stages": cfg.stages,
        "row_cost": cfg.row_cost,
        "schedule": cfg.schedule,
        "group_blocks": cfg.group_blocks,
        "ctas_per_sm": cfg.ctas_per_sm,
    }
