"""CUDA graph capture and replay of the package's operators.

The operators enqueue on the caller's stream and keep no host-side state that
a replay would miss (each launch leaves its workspace counters at zero), so a
captured SpMM replays correctly, including after its inputs change in place.
Warm-up runs on the capture stream first, as for any captured PyTorch code,
so that the workspace is allocated outside the capture.
"""

from __future__ import annotations

import pytest
import torch

from oracle import oracle
from kairo_b200.ops import KernelConfig, block_sparse_mm_bsr, bsr_from_tiles, sparse_gather, sparse_linear
from kairo_b200.types import SparseMask
from kairo_b200.workloads import WorkloadSpec, generate
from tests.conftest import rel_fro

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 1e-3


def _capture(fn):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        fn()
    return g


@pytest.mark.parametrize("case", [
    # dtype, bs, m, k, n, sparsity, mask, config
    (torch.float16, 32, 2048, 2048, 256, 0.95, "uniform", KernelConfig()),                    # rows
    (torch.float16, 16, 2048, 2048, 128, 0.99, "zipf", KernelConfig(num_ctas=5)),             # split rows
    (torch.bfloat16, 64, 512, 2048, 512, 0.8, "uniform", KernelConfig(schedule="bands")),     # bands
    (torch.float32, 16, 512, 512, 128, 0.8, "uniform", KernelConfig()),                       # SIMT
])
def test_spmm_graph_replay(case):
    dtype, bs, m, k, n, sp, mask, cfg = case
    p = generate(WorkloadSpec("g", dtype, m, k, n, bs, sp, mask=mask), seed=5)
    a = bsr_from_tiles(p.tiles.to(DEV), p.row_ids.to(DEV), p.col_ids.to(DEV), (m, k))
    b = p.b.to(DEV)
    out = torch.empty(m, n, dtype=torch.float32, device=DEV)
    g = _capture(lambda: block_sparse_mm_bsr(a, b, out=out, config=cfg))
    for trial in range(3):
        b2 = torch.randn(k, n, generator=torch.Generator().manual_seed(trial)).to(dtype)
        b.copy_(b2.to(DEV))
        out.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        ref = oracle.spmm_tiles(p.tiles, p.row_ids, p.col_ids, b2, m, k, n, bs)
        assert rel_fro(out, ref) <= TOL


def test_sparse_linear_graph_replay():
    spec = WorkloadSpec("g", torch.bfloat16, 512, 1024, 256, 64, 0.8, mask="magnitude", layout="linear",
                        a_std=0.02)
    p = generate(spec, seed=6)
    w = bsr_from_tiles(p.tiles.to(DEV), p.row_ids.to(DEV), p.col_ids.to(DEV), (spec.m, spec.k))
    x = p.b.to(DEV)
    y = torch.empty(spec.n, spec.m, dtype=torch.float32, device=DEV)
    g = _capture(lambda: sparse_linear(x, w, out=y))
    x2 = torch.randn(spec.n, spec.k, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16)
    x.copy_(x2.to(DEV))
    g.replay()
    torch.cuda.synchronize()
    ref = oracle.spmm_tiles(p.tiles, p.row_ids, p.col_ids, x2.t().contiguous(), spec.m, spec.k, spec.n, 64).t()
    assert rel_fro(y, ref) <= TOL


def test_sparse_gather_graph_replay():
    gen = torch.Generator().manual_seed(4)
    n, d = 1000, 64
    keep = torch.rand(n, d, generator=gen) < 0.3
    idx = keep.nonzero().t().contiguous()
    mask = SparseMask(indices=idx.to(DEV), values=torch.ones(idx.shape[1], device=DEV), dense_shape=(n, d),
                      sparsity_ratio=0.7)
    w = torch.randn(n, d, generator=gen).to(DEV)
    ids = torch.randint(0, n, (500,), generator=gen).to(DEV)
    holder = {}

    def step():
        holder["out"] = sparse_gather(w, mask, ids)

    g = _capture(step)
    ids2 = torch.randint(0, n, (500,), generator=gen)
    ids.copy_(ids2.to(DEV))
    g.replay()
    torch.cuda.synchronize()
    _, rs, cs = oracle.sort_coo_by_row(idx[0], idx[1], n)
    assert torch.equal(holder["out"].cpu(), oracle.sparse_gather(w.cpu(), oracle.row_offsets(rs, n), cs, ids2))


def test_sparse_scatter_grad_graph_replay():
    # A replay with new batch ids and gradients must clear and rewrite every
    # row (the clearing, key search, bucket sort and sums are all captured).
    from kairo_b200.ops import sparse_scatter_grad

    gen = torch.Generator().manual_seed(8)
    n, d, b = 5000, 64, 3000
    batch = torch.randint(0, n, (b,), generator=gen)
    active = torch.unique(batch)[::2].contiguous()
    grad = torch.randn(b, d, generator=gen).to(DEV)
    bid = batch.to(DEV)
    aid = active.to(DEV)
    holder = {}

    def step():
        holder["out"] = sparse_scatter_grad(grad, aid, bid, n, d)

    g = _capture(step)
    batch2 = torch.randint(0, n, (b,), generator=gen)
    grad2 = torch.randn(b, d, generator=gen)
    bid.copy_(batch2.to(DEV))
    grad.copy_(grad2.to(DEV))
    holder["out"].fill_(float("nan"))
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(holder["out"].cpu(), oracle.sparse_scatter_grad(grad2, active, batch2, n, d))


def test_split_bf16_graph_replay():
    # The opt-in split-bf16 path (split kernel + tcgen05 SpMM) captured and
    # replayed with new B values.
    p = generate(WorkloadSpec("g", torch.float32, 512, 512, 128, 16, 0.8), seed=7)
    a = bsr_from_tiles(p.tiles.to(DEV), p.row_ids.to(DEV), p.col_ids.to(DEV), (512, 512))
    b = p.b.to(DEV)
    out = torch.empty(512, 128, dtype=torch.float32, device=DEV)
    cfg = KernelConfig(kernel="split_bf16")
    g = _capture(lambda: block_sparse_mm_bsr(a, b, out=out, config=cfg))
    b2 = torch.randn(512, 128, generator=torch.Generator().manual_seed(11))
    b.copy_(b2.to(DEV))
    out.fill_(float("nan"))
    g.replay()
    torch.cuda.synchronize()
    ref = oracle.spmm_tiles(p.tiles, p.row_ids, p.col_ids, b2, 512, 512, 128, 16)
    assert rel_fro(out, ref) <= 1e-4
