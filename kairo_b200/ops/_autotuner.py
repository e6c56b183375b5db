"""Runtime tile / launch-shape selection for the block-sparse SpMM.

Keeps the reference's entry point and contract (kairo/ops/_autotuner.py:15-191):
``TileConfig``, ``CANDIDATE_CONFIGS``, ``DEFAULT_CONFIG``, ``BENCH_WARMUP``,
``BENCH_ITERS``, ``_cache_key``, and ``TileAutotuner.best_config(M, K, N,
sparsity)`` returning a dict with ``tile_m``, ``tile_n`` and ``tile_k``,
cached in ``TileAutotuner._cache`` and cleared by ``clear_cache()``.

On B200 the search space gains the Blackwell launch knobs of the tcgen05
kernel: ``n_tile`` (128 or 256 columns of C per work item, i.e. one or two
M=128 MMAs sharing each block), ``stages`` (shared-memory pipeline depth) and
``row_cost`` (scheduler weight of a block-row).  They are returned as extra
keys.  Timing uses CUDA events (median of ``BENCH_ITERS``) instead of host
wall-clock.  Without CUDA, ``best_config`` returns ``DEFAULT_CONFIG`` like the
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

    tile_m/tile_n/tile_k: the reference's keys; tile_m is the mask (block)
    granularity used for the timing run.  n_tile, stages, row_cost: tcgen05
    launch knobs (0 = library default).
    """

    tile_m: int
    tile_n: int
    tile_k: int
    n_tile: int = 0
    stages: int = 0
    row_cost: int = 0

    def __post_init__(self) -> None:
        if min(self.tile_m, self.tile_n, self.tile_k) <= 0:
            raise ValueError("tile sizes must be positive")
        if self.n_tile not in (0, 128, 256):
            raise ValueError("n_tile must be 0, 128 or 256")
        if self.stages < 0 or self.row_cost < 0:
            raise ValueError("stages and row_cost must be non-negative")


# Reference candidates (_autotuner.py:25-31), kept for the legacy keys.
CANDIDATE_CONFIGS: tuple[TileConfig, ...] = (
    TileConfig(tile_m=16, tile_n=16, tile_k=16),
    TileConfig(tile_m=32, tile_n=32, tile_k=16),
    TileConfig(tile_m=64, tile_n=64, tile_k=16),
    TileConfig(tile_m=16, tile_n=16, tile_k=32),
    TileConfig(tile_m=32, tile_n=32, tile_k=32),
)

DEFAULT_CONFIG = CANDIDATE_CONFIGS[0]

# Blackwell launch variants tried for 16-bit inputs on top of each tile size.
BLACKWELL_VARIANTS: tuple[tuple[int, int, int], ...] = (
    # (n_tile, stages, row_cost)
    (0, 0, 0),
    (128, 0, 0),
    (256, 0, 0),
    (128, 0, 4),
    (256, 4, 0),
)

BENCH_WARMUP = 2
BENCH_ITERS = 5


def _cache_key(M: int, K: int, N: int, sparsity: float, dtype: torch.dtype | None = None) -> str:
    """Bucketed key (dims to {128, 512, 2048, 4096}, sparsity to 0.1), plus dtype."""

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
    ) -> dict[str, Any]:
        """Best configuration for the problem size.

        Returns a dict with 'tile_m', 'tile_n', 'tile_k' (and the Blackwell
        keys 'n_tile', 'stages', 'row_cost').  Without CUDA, or if every
        candidate fails, the default config is returned.
        """
        key = _cache_key(M, K, N, sparsity, dtype)
        if key in self._cache:
            return self._cache[key]
        if not torch.cuda.is_available():
            result = _config_to_dict(DEFAULT_CONFIG)
            self._cache[key] = result
            return result
        best = self._benchmark(M, K, N, sparsity, dtype)
        self._cache[key] = best
        return best

    def _benchmark(self, M: int, K: int, N: int, sparsity: float, dtype: torch.dtype) -> dict[str, Any]:
        best_time = float("inf")
        best_cfg = DEFAULT_CONFIG
        for cfg in CANDIDATE_CONFIGS:
            if cfg.tile_m > M or cfg.tile_k > K:
                continue
            variants = BLACKWELL_VARIANTS if dtype in (torch.float16, torch.bfloat16) else ((0, 0, 0),)
            for n_tile, stages, row_cost in variants:
                cand = TileConfig(cfg.tile_m, cfg.tile_n, cfg.tile_k, n_tile, stages, row_cost)
                elapsed = self._time_config(cand, M, K, N, sparsity, dtype)
                if elapsed < best_time:
                    best_time = elapsed
                    best_cfg = cand
        return _config_to_dict(best_cfg)

    def _time_config(self, cfg: TileConfig, M: int, K: int, N: int, sparsity: float,
                     dtype: torch.dtype = torch.float32) -> float:
        """Median time in seconds of one BSR SpMM with ``cfg`` on random data
        at the given sparsity (a random tile mask of granularity tile_m)."""
        try:
            from kairo_b200.ops.spmm import KernelConfig, block_sparse_mm_bsr, bsr_from_tiles

            device = torch.device("cuda")
            tile = cfg.tile_m
            nbr = (M + tile - 1) // tile
            nbc = (K + tile - 1) // tile
            total = nbr * nbc
            nnz = max(1, int(total * (1.0 - sparsity)))
            perm = torch.randperm(total, device=device)[:nnz]
            rows = (perm // nbc).to(torch.int32)
            cols = (perm % nbc).to(torch.int32)
            tiles = torch.randn(nnz, tile, tile, device=device).to(dtype)
            B = torch.randn(K, N, device=device).to(dtype)
            a = bsr_from_tiles(tiles, rows, cols, (M, K))
            kc = KernelConfig(n_tile=cfg.n_tile, stages=cfg.stages, row_cost=cfg.row_cost)
            out = torch.empty(M, N, dtype=torch.float32, device=device)
            for _ in range(BENCH_WARMUP):
                block_sparse_mm_bsr(a, B, out=out, config=kc)
            torch.cuda.synchronize()
            times: list[float] = []
            for _ in range(BENCH_ITERS):
                start = torch.cuda.Event(enable_timing=True)
                end = torch.cuda.Event(enable_timing=True)
                start.record()
                block_sparse_mm_bsr(a, B, out=out, config=kc)
                end.record()
                end.synchronize()
                times.append(start.elapsed_time(end) / 1e3)
            times.sort()
            return times[len(times) // 2]
        except Exception as exc:  # noqa: BLE001 - a failing candidate is skipped, as in the reference
            _logger.debug("Autotuner config %s failed: %s", cfg, exc)
            return float("inf")

    def best_kernel_config(self, a, N: int, candidates=None):  # noqa: ANN001
        """Best :class:`KernelConfig` for an actual BlockSparseMatrix ``a``
        and N columns, timed on that matrix (CUDA events, median)."""
        from kairo_b200.ops.spmm import KernelConfig, block_sparse_mm_bsr

        key = f"bsr_{a.shape}_{a.block_size}_{a.nnzb}_{N}_{a.dtype}"
        if key in self._cache:
            return KernelConfig(**self._cache[key])
        if candidates is None:
            candidates = [KernelConfig(n_tile=nt, stages=st, row_cost=rc) for nt, st, rc in BLACKWELL_VARIANTS]
        B = torch.randn(a.shape[1], N, device=a.device).to(a.dtype)
        out = torch.empty(a.shape[0], N, dtype=torch.float32, device=a.device)
        best, best_t = KernelConfig(), float("inf")
        for kc in candidates:
            try:
                for _ in range(BENCH_WARMUP):
                    block_sparse_mm_bsr(a, B, out=out, config=kc)
                ts = []
                for _ in range(BENCH_ITERS):
                    s = torch.cuda.Event(enable_timing=True)
                    e = torch.cuda.Event(enable_timing=True)
                    s.record()
                    block_sparse_mm_bsr(a, B, out=out, config=kc)
                    e.record()
                    e.synchronize()
                    ts.append(s.elapsed_time(e))
                ts.sort()
                t = ts[len(ts) // 2]
            except Exception as exc:  # noqa: BLE001
                _logger.debug("kernel config %s failed: %s", kc, exc)
                continue
            if t < best_t:
                best, best_t = kc, t
        self._cache[key] = {"kernel": best.kernel, "n_tile": best.n_tile, "stages": best.stages,
                            "row_cost": best.row_cost, "num_ctas": best.num_ctas}
        return best

    def clear_cache(self) -> None:
        """Clear the autotuner cache."""
        self._cache.clear()


def _config_to_dict(cfg: TileConfig) -> dict[str, Any]:
    return {
        "tile_m": cfg.tile_m,
        "tile_n": cfg.tile_n,
        "tile_k": cfg.tile_k,
        "n_tile": cfg.n_tile,
        "stages": cfg.stages,
        "row_cost": cfg.row_cost,
    }
