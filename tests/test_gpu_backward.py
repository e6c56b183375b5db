"""Backward pass of the block-sparse linear layer against the CPU oracle.

* bsr_transpose: structure and transposed blocks bit-exact against the
  oracle's stable sort by block-column.
* dW (kairo_bsr_sddmm, tensor-core and CUDA-core kernels) and dX (the LINEAR
  SpMM on W^T): within the relative Frobenius bar TOL of the fp32 oracle.
* BlockSparseLinear: autograd gradients against the same references.
"""

from __future__ import annotations

import pytest
import torch

from oracle import oracle
from kairo_b200 import _lib
from kairo_b200.ops import (
    BlockSparseLinear,
    bsr_from_tiles,
    bsr_transpose,
    sparse_linear_backward,
    sparse_linear_weight_grad,
)
from kairo_b200.types import BlockSparseMatrix
from kairo_b200.workloads import WorkloadSpec, generate
from tests.conftest import rel_fro

pytestmark = pytest.mark.gpu

TOL = 1e-3
DEV = "cuda"


def _weight(dtype, m, k, bs, sp, seed, shuffle=False, mask="uniform"):
    spec = WorkloadSpec("w", dtype, m, k, 8, bs, sp, mask=mask, layout="linear", a_std=0.1)
    p = generate(spec, seed=seed)
    tiles, rows, cols = p.tiles, p.row_ids, p.col_ids
    if shuffle:
        g = torch.Generator().manual_seed(seed + 1)
        perm = torch.randperm(tiles.shape[0], generator=g)
        tiles, rows, cols = tiles[perm].contiguous(), rows[perm].contiguous(), cols[perm].contiguous()
    w = bsr_from_tiles(tiles.to(DEV), rows.to(DEV), cols.to(DEV), (m, k))
    return w, p


@pytest.mark.parametrize("case", [
    (torch.float32, 256, 384, 16, 0.7, False),
    (torch.float16, 512, 256, 32, 0.8, True),
    (torch.bfloat16, 640, 1024, 64, 0.85, False),
    (torch.bfloat16, 300, 200, 32, 0.6, True),      # ragged M, K
    (torch.float16, 64, 4096, 16, 0.0, False),      # dense block grid: long W^T rows
])
def test_transpose_bit_exact(case):
    dtype, m, k, bs, sp, shuffle = case
    w, _ = _weight(dtype, m, k, bs, sp, seed=3, shuffle=shuffle)
    t = bsr_transpose(w, check=True)
    rpt, cit, pt = oracle.bsr_transpose(w.row_ptr, w.col_idx, w.nbc)
    assert torch.equal(t.matrix.row_ptr.cpu(), rpt)
    assert torch.equal(t.matrix.col_idx.cpu(), cit)
    assert torch.equal(t.perm.cpu(), pt)
    stored = w.blocks if w.blk_idx is None else w.blocks[w.blk_idx.long()]
    assert torch.equal(t.matrix.blocks, stored[pt.to(DEV).long()].transpose(1, 2))
    assert t.matrix.shape == (k, m) and t.matrix.block_size == (bs, bs)
    assert t.matrix.max_row_blocks == int((rpt[1:] - rpt[:-1]).max())


def test_transpose_unaligned_blocks():
    """Blocks not 16-byte aligned take the element-wise transpose kernel."""
    w, _ = _weight(torch.bfloat16, 256, 512, 32, 0.7, seed=13)
    stored = w.blocks if w.blk_idx is None else w.blocks[w.blk_idx.long()]
    flat = torch.empty(stored.numel() + 1, dtype=stored.dtype, device=DEV)
    shifted = flat[1:].view(stored.shape)
    shifted.copy_(stored)
    ws = BlockSparseMatrix(row_ptr=w.row_ptr, col_idx=w.col_idx, blocks=shifted, shape=w.shape,
                           block_size=w.block_size)
    t = bsr_transpose(ws, check=True)
    _, _, pt = oracle.bsr_transpose(w.row_ptr, w.col_idx, w.nbc)
    assert torch.equal(t.matrix.blocks, stored[pt.to(DEV).long()].transpose(1, 2))


def test_transpose_empty_and_bad_index():
    w, _ = _weight(torch.float16, 128, 128, 32, 0.5, seed=4)
    e = BlockSparseMatrix(row_ptr=torch.zeros(w.nbr + 1, dtype=torch.int32, device=DEV),
                          col_idx=w.col_idx[:0], blocks=w.blocks[:0], shape=w.shape, block_size=w.block_size)
    t = bsr_transpose(e, check=True)
    assert int(t.matrix.row_ptr.abs().sum()) == 0 and t.matrix.nnzb == 0
    bad = w.col_idx.clone()
    bad[0] = w.nbc + 3
    wb = BlockSparseMatrix(row_ptr=w.row_ptr, col_idx=bad, blocks=w.blocks, shape=w.shape, block_size=w.block_size,
                           blk_idx=w.blk_idx)
    with pytest.raises(_lib.KairoDeviceError):
        bsr_transpose(wb, check=True)


SDD_CASES = [
    # dtype, m, k, n, bs, sparsity, out dtype    (bs 64 f16/bf16: tensor cores)
    (torch.bfloat16, 512, 1024, 256, 64, 0.8, torch.float32),
    (torch.float16, 640, 512, 200, 64, 0.7, torch.float32),      # batch not a multiple of 64
    (torch.bfloat16, 520, 600, 128, 64, 0.6, torch.bfloat16),    # ragged M, K; bf16 dW
    (torch.bfloat16, 256, 8192, 96, 64, 0.5, torch.float32),     # long columns of W^T
    (torch.float16, 256, 512, 100, 32, 0.8, torch.float32),      # CUDA cores
    (torch.float32, 128, 192, 70, 16, 0.6, torch.float32),       # fp32, CUDA cores
]


@pytest.mark.parametrize("case", SDD_CASES, ids=lambda c: f"{str(c[0])[6:]}-{c[1]}x{c[2]}-n{c[3]}-bs{c[4]}-"
                                                      f"{str(c[6])[6:]}")
def test_weight_grad_vs_oracle(case):
    dtype, m, k, n, bs, sp, odt = case
    w, _ = _weight(dtype, m, k, bs, sp, seed=7)
    g = torch.Generator().manual_seed(11)
    dy = torch.randn(n, m, generator=g).to(dtype)
    x = torch.randn(n, k, generator=g).to(dtype)
    dw = sparse_linear_weight_grad(dy.to(DEV), x.to(DEV), w, out_dtype=odt, check=True)
    ref = oracle.bsr_sddmm(w.row_ptr, w.col_idx, dy, x, bs, bs)
    if odt == torch.float32:
        assert rel_fro(dw, ref) <= TOL
    else:
        assert rel_fro(dw.float(), ref.to(odt).float()) <= TOL
    # a second call gives identical bits
    assert torch.equal(dw, sparse_linear_weight_grad(dy.to(DEV), x.to(DEV), w, out_dtype=odt))


@pytest.mark.parametrize("case", [(torch.bfloat16, 512, 1024, 256, 64, 0.8), (torch.float16, 384, 640, 130, 32, 0.7)])
def test_input_grad_vs_oracle(case):
    dtype, m, k, n, bs, sp = case
    w, p = _weight(dtype, m, k, bs, sp, seed=9, shuffle=True)
    g = torch.Generator().manual_seed(12)
    dy = torch.randn(n, m, generator=g).to(dtype)
    x = torch.randn(n, k, generator=g).to(dtype)
    dx, _ = sparse_linear_backward(dy.to(DEV), x.to(DEV), w, need_dw=False, check=True)
    # dX^T = W^T @ dY^T: the oracle on the transposed tile list
    ref = oracle.spmm_tiles(p.tiles.transpose(1, 2).contiguous(), p.col_ids, p.row_ids, dy.t().contiguous(), k, m, n,
                            bs).t()
    assert dx.dtype == dtype
    assert rel_fro(dx.float(), ref.to(dtype).float()) <= TOL


def test_block_sparse_linear_autograd():
    m, k, n, bs = 512, 1024, 192, 64
    w, p = _weight(torch.bfloat16, m, k, bs, 0.8, seed=21)
    layer = BlockSparseLinear(w)
    g = torch.Generator().manual_seed(22)
    x = torch.randn(n, k, generator=g).to(torch.bfloat16).to(DEV).requires_grad_(True)
    gy = torch.randn(n, m, generator=g).to(torch.bfloat16)
    y = layer(x)
    assert y.shape == (n, m) and y.dtype == torch.bfloat16
    y.backward(gy.to(DEV))
    # references: forward and both gradients from the oracle
    yref = oracle.spmm_tiles(p.tiles, p.row_ids, p.col_ids, x.detach().cpu().t().contiguous(), m, k, n, bs).t()
    assert rel_fro(y.detach().float(), yref.to(torch.bfloat16).float()) <= TOL
    dwref = oracle.bsr_sddmm(w.row_ptr, w.col_idx, gy, x.detach().cpu(), bs, bs)
    assert layer.blocks.grad.dtype == torch.bfloat16
    assert rel_fro(layer.blocks.grad.float(), dwref.to(torch.bfloat16).float()) <= TOL
    dxref = oracle.spmm_tiles(p.tiles.transpose(1, 2).contiguous(), p.col_ids, p.row_ids, gy.t().contiguous(), k, m,
                              n, bs).t()
    assert rel_fro(x.grad.float(), dxref.to(torch.bfloat16).float()) <= TOL
    # the weight changes, the cached structure of W^T follows the new values
    with torch.no_grad():
        layer.blocks.mul_(-2.0)
    x.grad = None
    layer(x).backward(gy.to(DEV))
    assert rel_fro(x.grad.float(), (dxref * -2.0).to(torch.bfloat16).float()) <= TOL


def test_weight_grad_large_batch():
    """A batch of 4096 rows (64 pipeline slabs per stack) on the tensor-core
    SDDMM."""
    m, k, n = 1024, 2048, 4096
    w, _ = _weight(torch.bfloat16, m, k, 64, 0.8, seed=5)
    dy = torch.randn(n, m, device=DEV).to(torch.bfloat16)
    x = torch.randn(n, k, device=DEV).to(torch.bfloat16)
    dw = sparse_linear_weight_grad(dy, x, w)
    ref = oracle.bsr_sddmm(w.row_ptr, w.col_idx, dy.cpu(), x.cpu(), 64, 64)
    assert rel_fro(dw, ref) <= TOL
