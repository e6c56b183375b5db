"""Block-sparse matrix multiplication on B200: operators over the C ABI.

``block_sparse_mm`` keeps the reference operator's signature, argument
checks and results (kairo/ops/spmm.py:58-105) and runs only on CUDA tensors:
the dense A is tiled by a device gather (replacing the per-tile host loop of
spmm.py:48-53), the tiles go through ``_C.acc_spmm_forward`` and the result is
fp32, as on the reference's CUDA path (csrc/acc_spmm_kernel.cu:169-170).

The BSR-level operators (``block_sparse_mm_bsr``, ``sparse_linear``) take a
:class:`~kairo_b200.types.BlockSparseMatrix` directly, for matrices whose
dense form does not fit in memory.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
from torch import Tensor

from kairo_b200 import _C, _lib
from kairo_b200.types import BlockSparseMatrix, SparseMask


@dataclass(frozen=True)
class KernelConfig:
    """Launch knobs of the BSR SpMM (0 = library default).

    kernel: "auto", "simt", "tcgen05" or "split_bf16" (opt-in, fp32 input:
    the tcgen05 kernel on a bf16 hi/lo split of A and B, hi·hi + hi·lo +
    lo·hi, about 2^-15 relative error per product); n_tile: C columns per work item on
    the tcgen05 kernel (128 or 256); stages: pipeline stages in shared
    memory; row_cost: scheduler weight of a block-row in units of one block
    (row-split schedule); num_ctas: persistent grid size; group_blocks:
    nonzero blocks loaded per pipeline stage (1..32); schedule: "auto",
    "rows" (block-rows split over CTAs, robust to skew) or "bands" (CTAs
    sweep B panels together, for a B slice larger than L2) or "groups"
    (row groups: block-rows of similar length taken ``group_rows`` at a time
    share each column's B panel and MMA; for skewed masks, STANDARD layout);
    band_rows: block-rows per band item; group_rows: block-rows per row group
    (2, 4 or 8; 0 = 4); ctas_per_sm: resident CTAs per SM of the
    row-split kernel (1..4), which share the SM's shared memory and TMEM so
    that one CTA's pipeline handoffs overlap another's MMAs.  Debugging knobs: wait_kcycles bounds every
    pipeline wait of the tcgen05 kernels (thousands of SM cycles; 0 = the
    default of about 4 s); debug_hold_stage=1 (a test hook) makes the
    row-split kernel hold back its first stage so that a bounded wait runs
    out and the launch reports a wait timeout instead of computing C.
    """

    kernel: str = "auto"
    n_tile: int = 0
    stages: int = 0
    row_cost: int = 0
    num_ctas: int = 0
    group_blocks: int = 0
    schedule: str = "auto"
    band_rows: int = 0
    wait_kcycles: int = 0
    debug_hold_stage: int = 0
    ctas_per_sm: int = 0
    group_rows: int = 0

    def __post_init__(self) -> None:
        if self.kernel not in ("auto", "simt", "tcgen05", "split_bf16"):
            raise ValueError(f"kernel must be 'auto', 'simt', 'tcgen05' or 'split_bf16', got {self.kernel!r}")
        if self.n_tile not in (0, 128, 256):
            raise ValueError(f"n_tile must be 0, 128 or 256, got {self.n_tile}")
        if self.schedule not in ("auto", "rows", "bands", "groups"):
            raise ValueError(f"schedule must be 'auto', 'rows', 'bands' or 'groups', got {self.schedule!r}")
        if self.group_rows not in (0, 2, 4, 8):
            raise ValueError(f"group_rows must be 0, 2, 4 or 8, got {self.group_rows}")
        if self.debug_hold_stage not in (0, 1):
            raise ValueError("debug_hold_stage must be 0 or 1")
        if self.ctas_per_sm > 4:
            raise ValueError("ctas_per_sm must be at most 4")
        for name in ("stages", "row_cost", "num_ctas", "group_blocks", "band_rows", "wait_kcycles", "ctas_per_sm"):
            if getattr(self, name) < 0:
                raise ValueError(f"{name} must be non-negative")
        if self.group_blocks > 32:
            raise ValueError("group_blocks must be at most 32")

    def to_c(self) -> _lib.KairoSpmmConfig:
        c = _lib.KairoSpmmConfig()
        c.kernel = {"auto": _lib.KERNEL_AUTO, "simt": _lib.KERNEL_SIMT, "tcgen05": _lib.KERNEL_TCGEN05,
                    "split_bf16": _lib.KERNEL_SPLIT_BF16}[self.kernel]
        c.n_tile = self.n_tile
        c.stages = self.stages
        c.row_cost = self.row_cost
        c.num_ctas = self.num_ctas
        c.group_blocks = self.group_blocks
        # Row groups have their own entry point; its other knobs are these.
        c.schedule = {"auto": _lib.SCHEDULE_AUTO, "rows": _lib.SCHEDULE_ROWS, "bands": _lib.SCHEDULE_BANDS,
                      "groups": _lib.SCHEDULE_AUTO}[self.schedule]
        c.band_rows = self.band_rows
        c.wait_kcycles = self.wait_kcycles
        c.debug_hold_stage = self.debug_hold_stage
        c.ctas_per_sm = self.ctas_per_sm
        return c


def pending_device_error(device: torch.device | int | None = None, clear: bool = True) -> int:
    """Device error word left by ``check=False`` launches on ``device``'s
    current stream (0 = none; KAIRO_DEVERR_* in the low 8 bits, the wait
    site above).  Synchronises that stream; ``clear`` resets the word."""
    return _lib.pending_device_error(device, clear)


def _require_cuda(*tensors: Tensor, op: str) -> None:
    for t in tensors:
        if not t.is_cuda:
            raise RuntimeError(f"kairo_b200.{op} runs on CUDA tensors only (got a {t.device} tensor); "
                               "this package has no CPU implementation")


def _dense_to_block_sparse(
    matrix: Tensor,
    block_mask: SparseMask,
    tile_size: int,
) -> tuple[Tensor, Tensor, Tensor]:
    """Dense matrix + tile mask -> (A_tiles, tile_row_ids, tile_col_ids).

    Same result as the reference (kairo/ops/spmm.py:16-55): tiles in mask
    order, zero-padded where a tile crosses the matrix edge, ids as int32.
    The tiles are gathered on the device by ``kairo_dense_to_tiles``.
    """
    _require_cuda(matrix, op="_dense_to_block_sparse")
    rows = block_mask.indices[0].to(device=matrix.device, dtype=torch.int32).contiguous()
    cols = block_mask.indices[1].to(device=matrix.device, dtype=torch.int32).contiguous()
    num_tiles = block_mask.nnz
    tiles = torch.empty(num_tiles, tile_size, tile_size, dtype=matrix.dtype, device=matrix.device)
    if num_tiles:
        a = matrix if matrix.stride(1) == 1 else matrix.contiguous()
        with torch.cuda.device(matrix.device):
            _lib.check(_lib.lib().kairo_dense_to_tiles(
                a.data_ptr(), a.shape[0], a.shape[1], a.stride(0), rows.data_ptr(), cols.data_ptr(), num_tiles,
                tile_size, _lib.kairo_dtype(a.dtype), tiles.data_ptr(), _lib.stream_handle(matrix.device)),
                "_dense_to_block_sparse")
    return tiles, rows, cols


def block_sparse_mm(
    A: Tensor,
    B: Tensor,
    block_mask: SparseMask,
    tile_size: int = 16,
    *,
    out_dtype: torch.dtype | None = None,
) -> Tensor:
    """Block-sparse matrix multiply: C = blocksparse(A) @ B.

    Only the tiles named by ``block_mask`` are read from A.  Mirrors the
    reference operator (kairo/ops/spmm.py:58-105) on CUDA tensors:
    raises ``ValueError("Inner dimensions must match: ...")`` on a K mismatch,
    returns zeros of A's dtype for an empty mask, and otherwise returns the
    fp32 product computed by the B200 kernels.

    Args:
        A: dense (M, K) matrix on a CUDA device.
        B: dense (K, N) matrix on the same device, same dtype as A.
        block_mask: SparseMask with tile-granular indices.
        tile_size: tile side length (default 16).
        out_dtype: None (the reference's fp32 result), torch.float32, or A's
            dtype: the fp32 accumulation rounded once.
    """
    M, K = A.shape
    K2, N = B.shape
    if K != K2:
        raise ValueError(f"Inner dimensions must match: A is ({M}, {K}), B is ({K2}, {N})")
    _require_cuda(A, B, op="block_sparse_mm")
    if out_dtype not in (None, torch.float32, A.dtype):
        raise TypeError("out_dtype must be None, torch.float32 or A's dtype")
    A_tiles, tile_row_ids, tile_col_ids = _dense_to_block_sparse(A, block_mask, tile_size)
    num_tiles = A_tiles.shape[0]
    if num_tiles == 0:
        return torch.zeros(M, N, dtype=out_dtype or A.dtype, device=A.device)
    C = _C.acc_spmm_forward(
        A_tiles.contiguous(),
        tile_row_ids.contiguous(),
        tile_col_ids.contiguous(),
        B.contiguous(),
        M, K, N, num_tiles, tile_size, tile_size,
    )
    return C if out_dtype in (None, torch.float32) else C.to(out_dtype)


def bsr_from_tiles(
    tiles: Tensor,
    tile_row_ids: Tensor,
    tile_col_ids: Tensor,
    shape: tuple[int, int],
) -> BlockSparseMatrix:
    """Builds a BlockSparseMatrix from a COO tile list, on the device.

    The block order is the reference's stable row sort
    (kairo/ops/sparse_embedding.py:49-56) with row offsets as in
    sparse_embedding.py:23-46; ``tiles`` stay where they are and ``blk_idx``
    maps BSR positions to them (``None`` when the list was already sorted).
    """
    _require_cuda(tiles, tile_row_ids, tile_col_ids, op="bsr_from_tiles")
    if tiles.dim() != 3:
        raise ValueError("tiles must be (num_tiles, bm, bk)")
    m, k = shape
    bm, bk = int(tiles.shape[1]), int(tiles.shape[2])
    nbr = (m + bm - 1) // bm
    nbc = (k + bk - 1) // bk
    nt = int(tiles.shape[0])
    dev = tiles.device
    rows = tile_row_ids.to(dtype=torch.int32).contiguous()
    cols = tile_col_ids.to(dtype=torch.int32).contiguous()
    if rows.numel() != nt or cols.numel() != nt:
        raise ValueError("tile id arrays must have one entry per tile")
    lib = _lib.lib()
    with torch.cuda.device(dev):
        row_ptr = torch.empty(nbr + 1, dtype=torch.int32, device=dev)
        col_idx = torch.empty(nt, dtype=torch.int32, device=dev)
        perm = torch.empty(nt, dtype=torch.int32, device=dev)
        nbytes = ctypes.c_size_t(0)
        _lib.check(lib.kairo_bsr_build_workspace_size(nt, nbr, ctypes.byref(nbytes)), "bsr_from_tiles")
        ws = torch.empty(max(nbytes.value, 256), dtype=torch.uint8, device=dev)
        ident = ctypes.c_int32(0)
        longest = ctypes.c_int32(0)
        _lib.check(lib.kairo_bsr_build(rows.data_ptr() if nt else None, cols.data_ptr() if nt else None, nt, nbr,
                                       nbc, row_ptr.data_ptr(), col_idx.data_ptr() if nt else None,
                                       perm.data_ptr() if nt else None, ctypes.byref(ident), ctypes.byref(longest),
                                       ws.data_ptr(), ws.numel(), _lib.stream_handle(dev)), "bsr_from_tiles")
    return BlockSparseMatrix(row_ptr=row_ptr, col_idx=col_idx, blocks=tiles.contiguous(), shape=(m, k),
                             block_size=(bm, bk), blk_idx=None if ident.value else perm,
                             max_row_blocks=int(longest.value))


def bsr_from_mask(A: Tensor, block_mask: SparseMask, tile_size: int) -> BlockSparseMatrix:
    """Dense A + tile mask -> BlockSparseMatrix (tiles gathered on the device)."""
    tiles, rows, cols = _dense_to_block_sparse(A, block_mask, tile_size)
    return bsr_from_tiles(tiles, rows, cols, (A.shape[0], A.shape[1]))


def _bsr_desc(a: BlockSparseMatrix) -> _lib.KairoBsr:
    d = _lib.KairoBsr()
    d.rows, d.cols = a.shape
    d.bm, d.bk = a.block_size
    d.nbr = a.nbr
    d.nnzb = a.nnzb
    d.nblocks_stored = int(a.blocks.shape[0])
    d.row_ptr = a.row_ptr.data_ptr()
    d.col_idx = a.col_idx.data_ptr() if a.nnzb else None
    d.blk_idx = a.blk_idx.data_ptr() if a.blk_idx is not None and a.nnzb else None
    d.blocks = a.blocks.data_ptr() if a.blocks.numel() else None
    d.dtype = _lib.kairo_dtype(a.dtype)
    d.max_row_blocks = a.max_row_blocks
    return d


class RowGroups:
    """Row groups of a BSR matrix on its device (``kairo_bsr_stack_build``).

    The block-rows, ordered by block count (longest first), are taken
    ``rows_per_group`` at a time; each group's distinct column-blocks are its
    stacked blocks.  Built once per matrix structure (it synchronises the
    current stream once) and reused by every SpMM on that matrix.
    """

    def __init__(self, a: BlockSparseMatrix, rows_per_group: int) -> None:
        lib = _lib.lib()
        desc = _bsr_desc(a)
        nbytes = ctypes.c_size_t(0)
        with torch.cuda.device(a.device):
            _lib.check(lib.kairo_bsr_stack_size(ctypes.byref(desc), rows_per_group, ctypes.byref(nbytes)),
                       "kairo_bsr_stack_size")
            self.mem = torch.empty(max(int(nbytes.value), 4), dtype=torch.uint8, device=a.device)
            self.desc = _lib.KairoBsrStack()
            _lib.check(lib.kairo_bsr_stack_build(ctypes.byref(desc), rows_per_group, self.mem.data_ptr(),
                                                 self.mem.numel(), ctypes.byref(self.desc),
                                                 _lib.stream_handle(a.device)), "kairo_bsr_stack_build")
        self.rows_per_group = rows_per_group
        self.ngroups = int(self.desc.ngroups)
        self.nsuper = int(self.desc.nsuper)

    def tables(self) -> dict[str, Tensor]:
        """The group tables as int32 tensors viewing the group memory."""
        d = self.desc
        base = self.mem.data_ptr()
        words = self.mem.view(torch.int32)

        def view(ptr: int, count: int) -> Tensor:
            off = (ptr - base) // 4
            return words[off:off + count]

        g, r, ns = self.ngroups, self.rows_per_group, self.nsuper
        return {"row_map": view(d.row_map, g * r), "group_ptr": view(d.group_ptr, g + 1),
                "super_col": view(d.super_col, ns), "super_mask": view(d.super_mask, ns),
                "super_blk": view(d.super_blk, ns * r)}


def bsr_row_groups(a: BlockSparseMatrix, rows_per_group: int = 4) -> RowGroups:
    """The :class:`RowGroups` of ``a`` with ``rows_per_group`` rows (cached
    on the matrix: its row_ptr / col_idx / blk_idx do not change)."""
    cache = a.__dict__.get("_row_groups")
    if cache is None:
        cache = {}
        object.__setattr__(a, "_row_groups", cache)
    if rows_per_group not in cache:
        cache[rows_per_group] = RowGroups(a, rows_per_group)
    return cache[rows_per_group]


# Automatic row groups: only for masks whose longest block-row is far above
# the mean (a skewed mask), and only when grouping leaves at most this many
# stacked blocks per block (each stacked block costs one B panel load).
_GROUPS_MIN_SKEW = 8.0
_GROUPS_MAX_RATIO = 0.6
# Whether AUTO may take row groups at all (see the kernel notes: on the
# measured skewed workload they do not yet beat the row-split schedule).
_GROUPS_AUTO = False


def _row_groups_for(a: BlockSparseMatrix, layout: int, config: KernelConfig | None) -> RowGroups | None:
    cfg = config or KernelConfig()
    rg = cfg.group_rows or 4
    if cfg.schedule == "groups":
        if layout != _lib.LAYOUT_STANDARD:
            raise ValueError("the row-group schedule implements the STANDARD layout (block_sparse_mm_bsr) only")
        return bsr_row_groups(a, rg)
    if (not _GROUPS_AUTO or cfg.schedule != "auto" or cfg.kernel not in ("auto", "tcgen05")
            or layout != _lib.LAYOUT_STANDARD):
        return None
    bm, bk = a.block_size
    if (a.dtype not in (torch.float16, torch.bfloat16) or bm != bk or bm not in (16, 32) or a.nnzb == 0
            or a.nbr > 16384 or a.nbc > 16384 or cfg.ctas_per_sm or cfg.num_ctas):
        return None
    mean = a.nnzb / max(a.nbr, 1)
    if a.max_row_blocks < max(64.0, _GROUPS_MIN_SKEW * mean):
        return None
    choice = a.__dict__.get("_auto_groups", {})
    if rg not in choice:
        try:
            groups = bsr_row_groups(a, rg)
            choice[rg] = groups if groups.nsuper <= _GROUPS_MAX_RATIO * a.nnzb else None
        except _lib.KairoError:
            choice[rg] = None
        object.__setattr__(a, "_auto_groups", choice)
    return choice[rg]


def describe(a: BlockSparseMatrix, n: int, *, linear: bool = False, config: KernelConfig | None = None) -> dict:
    """What ``block_sparse_mm_bsr`` (``linear=False``) or ``sparse_linear``
    (``linear=True``, N = rows of X) would run for ``a``: kernel, schedule,
    kernel launches per call, grid and pipeline shape, workspace bytes."""
    lib = _lib.lib()
    plan = _lib.KairoSpmmPlan()
    desc = _bsr_desc(a)
    cfg = (config or KernelConfig()).to_c()
    layout = _lib.LAYOUT_LINEAR if linear else _lib.LAYOUT_STANDARD
    groups = _row_groups_for(a, layout, config)
    with torch.cuda.device(a.device):
        if groups is not None:
            _lib.check(lib.kairo_bsr_spmm_stacked_describe(ctypes.byref(desc), ctypes.byref(groups.desc), int(n),
                                                           ctypes.byref(cfg), ctypes.byref(plan)), "describe")
        else:
            _lib.check(lib.kairo_bsr_spmm_describe(ctypes.byref(desc), layout, int(n), ctypes.byref(cfg),
                                                   ctypes.byref(plan)), "describe")
    kernel = {0: "none", _lib.KERNEL_SIMT: "simt", _lib.KERNEL_TCGEN05: "tcgen05",
              _lib.KERNEL_SPLIT_BF16: "split_bf16"}[plan.kernel]
    schedule = {0: "none", _lib.SCHEDULE_ROWS: "rows", _lib.SCHEDULE_BANDS: "bands",
                _lib.SCHEDULE_GROUPS: "groups"}[plan.schedule]
    out = {"kernel": kernel, "schedule": schedule, "launches": plan.launches, "grid": plan.grid,
           "n_tile": plan.n_tile, "stages": plan.stages, "group_blocks": plan.group_blocks, "rows": plan.rows,
           "workspace_bytes": int(plan.workspace_bytes)}
    if groups is not None:
        out["stacked_blocks"] = groups.nsuper
    return out


def _launch(a: BlockSparseMatrix, b: Tensor, ldb: int, layout: int, n: int, out: Tensor, ldc: int,
            config: KernelConfig | None, check_device: bool) -> None:
    lib = _lib.lib()
    desc = _bsr_desc(a)
    cfg = (config or KernelConfig()).to_c()
    dev = a.device
    groups = _row_groups_for(a, layout, config)
    if groups is not None and (config is None or config.schedule != "groups") and (ldb % 8 or b.data_ptr() % 16):
        groups = None  # the row-group kernel copies B with TMA: 16-byte rows only
    name = "kairo_bsr_spmm_stacked" if groups is not None else "kairo_bsr_spmm"
    with torch.cuda.device(dev):
        nbytes = ctypes.c_size_t(0)
        if groups is not None:
            _lib.check(lib.kairo_bsr_spmm_stacked_workspace_size(ctypes.byref(desc), ctypes.byref(groups.desc), n,
                                                                 ctypes.byref(cfg), ctypes.byref(nbytes)), name)
        else:
            _lib.check(lib.kairo_bsr_spmm_workspace_size(ctypes.byref(desc), layout, n, ctypes.byref(cfg),
                                                         ctypes.byref(nbytes)), name)
        ws = _lib.workspace(nbytes.value, dev)
        if check_device:
            _lib.take_pending_error(ws, name)
        if groups is not None:
            _lib.check(lib.kairo_bsr_spmm_stacked(ctypes.byref(desc), ctypes.byref(groups.desc), b.data_ptr(), ldb, n,
                                                  out.data_ptr(), ldc, ctypes.byref(cfg), ws.data_ptr(), ws.numel(),
                                                  _lib.stream_handle(dev)), name)
        else:
            _lib.check(lib.kairo_bsr_spmm(ctypes.byref(desc), b.data_ptr(), ldb, layout, n, out.data_ptr(), ldc,
                                          _lib.kairo_dtype(out.dtype), ctypes.byref(cfg), ws.data_ptr(), ws.numel(),
                                          _lib.stream_handle(dev)), name)
        if check_device:
            _lib.raise_on_device_error(ws)


def block_sparse_mm_bsr(
    a: BlockSparseMatrix,
    B: Tensor,
    *,
    out: Tensor | None = None,
    config: KernelConfig | None = None,
    check: bool = False,
) -> Tensor:
    """C = A_bsr @ B in fp32 (B: (K, N), same dtype as the blocks).

    Every element of C is written.  ``check=True`` synchronises and raises
    :class:`~kairo_b200._lib.KairoDeviceError` if the device recorded an
    error in this launch (an out-of-range block index or a pipeline wait
    that timed out).  With ``check=False`` (asynchronous) such errors stay
    in the stream's workspace until :func:`pending_device_error` reads them;
    the next ``check=True`` launch takes them out first and reports them as
    a :class:`~kairo_b200._lib.KairoDeviceWarning`, not as its own.
    """
    _require_cuda(a.blocks, B, op="block_sparse_mm_bsr")
    m, k = a.shape
    if B.dim() != 2 or B.shape[0] != k:
        raise ValueError(f"Inner dimensions must match: A is ({m}, {k}), B is {tuple(B.shape)}")
    if B.dtype != a.dtype:
        raise TypeError(f"B dtype {B.dtype} differs from block dtype {a.dtype}")
    if B.stride(1) != 1:
        B = B.contiguous()
    n = B.shape[1]
    if out is None:
        out = torch.empty(m, n, dtype=torch.float32, device=B.device)
    elif out.shape != (m, n) or out.dtype != torch.float32 or out.stride(1) != 1:
        raise ValueError("out must be a row-major (M, N) float32 tensor")
    _launch(a, B, B.stride(0), _lib.LAYOUT_STANDARD, n, out, out.stride(0), config, check)
    return out


def sparse_linear(
    X: Tensor,
    W: BlockSparseMatrix,
    *,
    out_dtype: torch.dtype | None = None,
    out: Tensor | None = None,
    config: KernelConfig | None = None,
    check: bool = False,
) -> Tensor:
    """Y = X @ W^T for a block-sparse weight W (out_features x in_features).

    X: (batch, in_features), same dtype as W's blocks.  Y: (batch,
    out_features) in ``out_dtype`` (default: X's dtype), accumulated in fp32
    and rounded once.  This is ``block_sparse_mm`` with B = X^T and C = Y^T,
    computed without transposing X or Y.
    """
    _require_cuda(W.blocks, X, op="sparse_linear")
    m, k = W.shape
    if X.dim() != 2 or X.shape[1] != k:
        raise ValueError(f"Inner dimensions must match: X is {tuple(X.shape)}, W is ({m}, {k})")
    if X.dtype != W.dtype:
        raise TypeError(f"X dtype {X.dtype} differs from weight dtype {W.dtype}")
    if X.stride(1) != 1:
        X = X.contiguous()
    n = X.shape[0]
    odt = out_dtype or X.dtype
    if out is None:
        out = torch.empty(n, m, dtype=odt, device=X.device)
    elif out.shape != (n, m) or out.stride(1) != 1:
        raise ValueError("out must be a row-major (batch, out_features) tensor")
    _launch(W, X, X.stride(0), _lib.LAYOUT_LINEAR, n, out, out.stride(0), config, check)
    return out
