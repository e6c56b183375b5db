"""Seeded synthetic block-sparse SpMM problems and their roofline accounting.

Five named problem families (sizes can be scaled down for tests):

  fp32_uniform      A 4096x4096, 16x16 blocks, 90% block sparsity, N(0,1); B 4096x256
  fp16_uniform      A 16384x16384, 32x32 blocks, 95%, N(0,0.02^2); B 16384x512 N(0,1)
  bf16_linear       W 8192x32768 (out x in), 64x64 blocks, top-20% blocks by L2 norm
                    of an N(0,0.02^2) init; X 8192x32768 N(0,1); Y = X W^T in bf16
  fp16_zipf         A 65536x65536, 16x16 blocks, 99%, per-row block counts Zipf(1.1)
                    (load-imbalance case); B 65536x128
  bf16_uniform      A 262144x262144, 32x32 blocks, 99.5%, N(0,0.02^2); B 262144x1024

Uniform masks follow the reference's test generator (tests/ops/test_spmm_ops.py:
21-44): ``manual_seed(seed)``, ``randperm(total)[:nnz]`` with
``nnz = max(1, int(total * (1 - sparsity)))``, rows/cols by division, stable
sort by row.  The magnitude-pruned mask keeps the top-k block norms and sorts
the kept indices (the convention of kairo/training/sparse_rec/topology.py:
95-96).  The Zipf mask is this package's own construction (see zipf_counts).
Draw order: mask, then block values, then B.
"""

from __future__ import annotations

from dataclasses import dataclass, replace

import numpy as np
import torch

from kairo_b200.types import SparseMask


@dataclass(frozen=True)
class WorkloadSpec:
    name: str
    dtype: torch.dtype
    m: int
    k: int
    n: int
    block: int
    sparsity: float
    mask: str = "uniform"       # uniform | zipf | magnitude
    layout: str = "standard"    # standard: C = A B ; linear: Y = X A^T
    a_std: float = 1.0
    b_std: float = 1.0
    out_dtype: torch.dtype = torch.float32

    @property
    def nbr(self) -> int:
        return (self.m + self.block - 1) // self.block

    @property
    def nbc(self) -> int:
        return (self.k + self.block - 1) // self.block

    @property
    def nnzb(self) -> int:
        total = self.nbr * self.nbc
        return max(1, int(total * (1.0 - self.sparsity)))

    def scaled(self, m: int, k: int, n: int) -> "WorkloadSpec":
        return replace(self, name=f"{self.name}@{m}x{k}x{n}", m=m, k=k, n=n)


WORKLOADS: dict[str, WorkloadSpec] = {
    "fp32_uniform": WorkloadSpec("fp32_uniform", torch.float32, 4096, 4096, 256, 16, 0.90),
    "fp16_uniform": WorkloadSpec("fp16_uniform", torch.float16, 16384, 16384, 512, 32, 0.95, a_std=0.02),
    "bf16_linear": WorkloadSpec("bf16_linear", torch.bfloat16, 8192, 32768, 8192, 64, 0.80, mask="magnitude",
                                layout="linear", a_std=0.02, out_dtype=torch.bfloat16),
    "fp16_zipf": WorkloadSpec("fp16_zipf", torch.float16, 65536, 65536, 128, 16, 0.99, mask="zipf"),
    "bf16_uniform": WorkloadSpec("bf16_uniform", torch.bfloat16, 262144, 262144, 1024, 32, 0.995, a_std=0.02),
}


@dataclass
class Problem:
    """One generated problem.  Blocks are in mask order (row-sorted)."""

    spec: WorkloadSpec
    mask: SparseMask            # tile-level COO, int64 indices
    tiles: torch.Tensor         # (nnzb, bs, bs) in spec.dtype
    b: torch.Tensor             # B (k x n) for standard, X (n x k) for linear

    @property
    def row_ids(self) -> torch.Tensor:
        return self.mask.indices[0].to(torch.int32)

    @property
    def col_ids(self) -> torch.Tensor:
        return self.mask.indices[1].to(torch.int32)


def uniform_mask(nbr: int, nbc: int, sparsity: float, gen: torch.Generator, device) -> SparseMask:
    total = nbr * nbc
    nnz = max(1, int(total * (1.0 - sparsity)))
    perm = torch.randperm(total, generator=gen, device=device)[:nnz]
    rows = perm // nbc
    cols = perm % nbc
    order = torch.argsort(rows, stable=True)
    indices = torch.stack([rows[order], cols[order]]).to(torch.int64)
    return SparseMask(indices=indices, values=torch.ones(nnz, device=device), dense_shape=(nbr, nbc),
                      sparsity_ratio=sparsity)


def zipf_counts(nbr: int, nbc: int, nnz: int, seed: int, s: float = 1.1) -> np.ndarray:
    """Blocks per block-row: Zipf(s) draws rescaled to sum to ``nnz`` with at
    most ``nbc`` blocks per row.

    1. raw = numpy.random.default_rng(seed).zipf(s, nbr) (float64).
    2. Water-filling cap: while some uncapped row's proportional share
       raw_i * remaining / sum(raw of uncapped rows) exceeds nbc, fix every
       such row at nbc and remove it.
    3. The uncapped rows get floor(share); the leftover blocks go one each to
       the rows with the largest fractional parts (ties: lower row index),
       skipping rows already at nbc.
    """
    if nnz > nbr * nbc:
        raise ValueError("nnz exceeds the block grid")
    raw = np.random.default_rng(seed).zipf(s, nbr).astype(np.float64)
    counts = np.zeros(nbr, dtype=np.int64)
    active = np.ones(nbr, dtype=bool)
    remaining = nnz
    while True:
        tot = raw[active].sum()
        share = np.zeros(nbr)
        share[active] = raw[active] * remaining / tot
        over = active & (share > nbc)
        if not over.any():
            break
        counts[over] = nbc
        remaining -= nbc * int(over.sum())
        active &= ~over
    base = np.floor(share).astype(np.int64)
    counts[active] = base[active]
    left = nnz - int(counts.sum())
    frac = share - base
    order = np.lexsort((np.arange(nbr), -frac))  # largest fraction first, then lower index
    for i in order:
        if left == 0:
            break
        if active[i] and counts[i] < nbc:
            counts[i] += 1
            left -= 1
    if left:
        raise RuntimeError("could not place every block")
    return counts


def zipf_mask(nbr: int, nbc: int, sparsity: float, seed: int, gen: torch.Generator, device) -> SparseMask:
    nnz = max(1, int(nbr * nbc * (1.0 - sparsity)))
    counts = zipf_counts(nbr, nbc, nnz, seed)
    rows, cols = [], []
    for r in np.nonzero(counts)[0]:
        c = int(counts[r])
        pick = torch.randperm(nbc, generator=gen)[:c].sort().values
        rows.append(torch.full((c,), int(r), dtype=torch.int64))
        cols.append(pick.to(torch.int64))
    indices = torch.stack([torch.cat(rows), torch.cat(cols)]).to(device)
    return SparseMask(indices=indices, values=torch.ones(nnz, device=device), dense_shape=(nbr, nbc),
                      sparsity_ratio=sparsity)


def generate(spec: WorkloadSpec, seed: int = 0, device: str | torch.device = "cpu") -> Problem:
    """Deterministic problem for (spec, seed, device type).  CPU and CUDA
    generators produce different streams; each caller uses one device."""
    device = torch.device(device)
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    bs = spec.block
    if spec.mask == "magnitude":
        # W values first (the mask is a function of them), blocks kept by norm.
        w = torch.randn(spec.m, spec.k, generator=gen, device=device) * spec.a_std
        nbr, nbc = spec.nbr, spec.nbc
        if spec.m % bs or spec.k % bs:
            raise ValueError("magnitude-pruned workloads need block-aligned shapes")
        norms = w.view(nbr, bs, nbc, bs).permute(0, 2, 1, 3).reshape(nbr * nbc, bs * bs).norm(dim=1)
        keep = norms.topk(spec.nnzb, largest=True).indices.sort().values
        rows, cols = keep // nbc, keep % nbc
        tiles = w.view(nbr, bs, nbc, bs)[rows, :, cols, :].to(spec.dtype).contiguous()
        del w
        mask = SparseMask(indices=torch.stack([rows, cols]).to(torch.int64), values=torch.ones(keep.numel(), device=device),
                          dense_shape=(nbr, nbc), sparsity_ratio=spec.sparsity)
    else:
        if spec.mask == "uniform":
            mask = uniform_mask(spec.nbr, spec.nbc, spec.sparsity, gen, device)
        elif spec.mask == "zipf":
            mask = zipf_mask(spec.nbr, spec.nbc, spec.sparsity, seed, gen if device.type == "cpu" else
                             torch.Generator().manual_seed(seed), device)
        else:
            raise ValueError(f"unknown mask kind {spec.mask}")
        tiles = (torch.randn(mask.nnz, bs, bs, generator=gen, device=device) * spec.a_std).to(spec.dtype)
        # Zero the parts of edge tiles that lie outside the matrix, as the
        # reference's tiling does (kairo/ops/spmm.py:43-53).
        if spec.m % bs or spec.k % bs:
            r0 = mask.indices[0] * bs
            c0 = mask.indices[1] * bs
            ii = torch.arange(bs, device=device)
            rv = (r0[:, None] + ii[None, :]) < spec.m
            cv = (c0[:, None] + ii[None, :]) < spec.k
            inside = rv[:, :, None] & cv[:, None, :]
            tiles = torch.where(inside, tiles, torch.zeros((), dtype=tiles.dtype, device=device))
    if spec.layout == "linear":
        b = (torch.randn(spec.n, spec.k, generator=gen, device=device) * spec.b_std).to(spec.dtype)
    else:
        b = (torch.randn(spec.k, spec.n, generator=gen, device=device) * spec.b_std).to(spec.dtype)
    return Problem(spec=spec, mask=mask, tiles=tiles, b=b)


# ------------------------------------------------------------------ accounting

def _esize(dt: torch.dtype) -> int:
    return torch.tensor([], dtype=dt).element_size()


def flops(spec: WorkloadSpec, nnzb: int | None = None) -> float:
    """Nonzero-block FLOPs: 2 * nnzb * bm * bk * N."""
    nnzb = spec.nnzb if nnzb is None else nnzb
    return 2.0 * nnzb * spec.block * spec.block * spec.n


def canonical_bytes(spec: WorkloadSpec, nnzb: int | None = None, nbr: int | None = None,
                    m: int | None = None) -> float:
    """A blocks + int32 indices (col_idx + row_ptr) + the gathered B panel of
    every block (bk x N each) + C."""
    nnzb = spec.nnzb if nnzb is None else nnzb
    nbr = spec.nbr if nbr is None else nbr
    m = spec.m if m is None else m
    sa = _esize(spec.dtype)
    sc = _esize(spec.out_dtype)
    return (nnzb * spec.block * spec.block * sa + (nnzb + nbr + 1) * 4 + nnzb * spec.block * spec.n * sa
            + m * spec.n * sc)


def strict_bytes(spec: WorkloadSpec, nnzb: int | None = None, nbr: int | None = None,
                 m: int | None = None) -> float:
    """As canonical_bytes, but B counted once (K x N)."""
    nnzb = spec.nnzb if nnzb is None else nnzb
    nbr = spec.nbr if nbr is None else nbr
    m = spec.m if m is None else m
    sa = _esize(spec.dtype)
    sc = _esize(spec.out_dtype)
    return nnzb * spec.block * spec.block * sa + (nnzb + nbr + 1) * 4 + spec.k * spec.n * sa + m * spec.n * sc


def roofline_time(flop: float, nbytes: float, tflops: float, gbs: float) -> float:
    """max(FLOP / peak, bytes / bandwidth) in seconds."""
    return max(flop / (tflops * 1e12), nbytes / (gbs * 1e9))



# ------------------------------------------------------------------ checking

def block_row_errors(c: torch.Tensor, ref: torch.Tensor, bm: int, chunk_rows: int = 1 << 16) -> torch.Tensor:
    """Relative Frobenius error of every block-row of ``c`` against ``ref``.

    Both are (M, N); block-row i is rows i*bm .. (i+1)*bm.  Computed on the
    host in float64, ``chunk_rows`` rows at a time, so that a 262144 x 1024
    result needs no float64 copy of the whole matrix.  A block-row whose
    reference is all zero reports its absolute error norm instead.
    Returns a float64 tensor of ceil(M / bm) errors.
    """
    if c.shape != ref.shape:
        raise ValueError(f"shape mismatch {tuple(c.shape)} vs {tuple(ref.shape)}")
    m = c.shape[0]
    nbr = (m + bm - 1) // bm
    num = torch.zeros(nbr, dtype=torch.float64)
    den = torch.zeros(nbr, dtype=torch.float64)
    step = max(bm, chunk_rows // bm * bm)
    for r0 in range(0, m, step):
        r1 = min(m, r0 + step)
        x = c[r0:r1].detach().to("cpu", torch.float64)
        y = ref[r0:r1].detach().to("cpu", torch.float64)
        d2 = (x - y).square().sum(dim=1)
        y2 = y.square().sum(dim=1)
        rows = torch.arange(r0, r1) // bm
        num.index_add_(0, rows, d2)
        den.index_add_(0, rows, y2)
    return torch.where(den > 0, (num / den.clamp_min(1e-300)).sqrt(), num.sqrt())


def rel_fro_chunked(c: torch.Tensor, ref: torch.Tensor, chunk_rows: int = 1 << 16) -> float:
    """||c - ref||_F / ||ref||_F in float64, ``chunk_rows`` rows at a time."""
    num = den = 0.0
    for r0 in range(0, c.shape[0], chunk_rows):
        x = c[r0:r0 + chunk_rows].detach().to("cpu", torch.float64)
        y = ref[r0:r0 + chunk_rows].detach().to("cpu", torch.float64)
        num += float((x - y).square().sum())
        den += float(y.square().sum())
    return (num / den) ** 0.5 if den > 0 else num ** 0.5
