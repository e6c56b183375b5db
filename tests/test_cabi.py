"""The C-ABI library: it loads, exports every entry point the header declares,
and its host-only paths (status strings, size queries, argument validation,
the row partition) behave as documented.  No device work is launched."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from kairo_b200 import _build, _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "kairo_spmm.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"KAIRO_API\s+[\w\s\*]+?\b(kairo_\w+)\s*\(", text)))


def test_library_builds_for_sm100a_and_loads():
    assert "arch=compute_100a,code=sm_100a" in " ".join(_build.ARCH_FLAGS)
    lib = _lib.lib()
    assert lib.kairo_abi_version() == _lib.ABI_VERSION == 2


def test_every_declared_symbol_is_exported():
    names = declared_symbols()
    assert len(names) >= 12
    lib = ctypes.CDLL(str(_build.LIB))
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(_lib.EXPORTED_SYMBOLS)


def test_status_strings():
    lib = _lib.lib()
    assert lib.kairo_status_string(0) == b"success"
    assert lib.kairo_status_string(2) == b"not supported"
    assert lib.kairo_status_string(99) == b"unknown status"


def test_workspace_size_queries():
    lib = _lib.lib()
    n = ctypes.c_size_t(0)
    assert lib.kairo_bsr_build_workspace_size(1000, 64, ctypes.byref(n)) == 0 and n.value >= 256
    assert lib.kairo_acc_spmm_forward_workspace_size(512, 512, 256, 100, 32, 32, _lib.DTYPE_F16,
                                                     ctypes.byref(n)) == 0
    assert n.value > 128 * 1024  # includes the split-row counter banks
    assert lib.kairo_acc_spmm_forward_workspace_size(0, 512, 256, 100, 32, 32, _lib.DTYPE_F16,
                                                     ctypes.byref(n)) == _lib.INVALID_VALUE
    assert b"positive" in lib.kairo_last_error_message()
    d = _lib.KairoBsr(rows=4096, cols=4096, bm=32, bk=32, nbr=128, nnzb=1000, nblocks_stored=1000,
                      dtype=_lib.DTYPE_BF16)
    assert lib.kairo_bsr_spmm_workspace_size(ctypes.byref(d), 0, 512, None, ctypes.byref(n)) == 0
    assert n.value > 128 * 1024


def test_bsr_spmm_rejects_bad_descriptors_before_launch():
    lib = _lib.lib()
    d = _lib.KairoBsr(rows=100, cols=64, bm=16, bk=16, nbr=6, nnzb=1, nblocks_stored=1, dtype=_lib.DTYPE_F16)
    st = lib.kairo_bsr_spmm(ctypes.byref(d), None, 64, 0, 64, None, 64, 0, None, None, 0, None)
    assert st == _lib.INVALID_VALUE
    assert b"nbr" in lib.kairo_last_error_message()
    d.nbr = 7
    d.dtype = 9
    assert lib.kairo_bsr_spmm(ctypes.byref(d), None, 64, 0, 64, None, 64, 0, None, None, 0, None) == _lib.INVALID_VALUE
    d.dtype = _lib.DTYPE_F16
    assert lib.kairo_bsr_spmm(ctypes.byref(d), None, 64, 5, 64, None, 64, 0, None, None, 0, None) == _lib.INVALID_VALUE
    # an empty problem (no rows) is a no-op that succeeds without touching a device
    d0 = _lib.KairoBsr(rows=0, cols=64, bm=16, bk=16, nbr=0, nnzb=0, nblocks_stored=0, dtype=_lib.DTYPE_F16)
    assert lib.kairo_bsr_spmm(ctypes.byref(d0), None, 64, 0, 64, None, 64, 0, None, None, 0, None) == 0


def _lower_bound_partition(row_ptr: np.ndarray, parts: int) -> list[int]:
    nnz = int(row_ptr[-1])
    nbr = len(row_ptr) - 1
    out = [0]
    for p in range(1, parts):
        r = int(np.searchsorted(row_ptr, nnz * p // parts, side="left"))
        out.append(min(max(r, out[-1]), nbr))
    out.append(nbr)
    return out


@pytest.mark.parametrize("parts", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_partition_rows(parts, seed):
    rng = np.random.default_rng(seed)
    counts = rng.integers(0, 50, size=200)
    counts[rng.integers(0, 200, size=5)] = 0
    rp = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
    from kairo_b200.sharding import partition_rows
    import torch

    b = partition_rows(torch.from_numpy(rp), parts)
    assert b == _lower_bound_partition(rp, parts)
    assert b[0] == 0 and b[-1] == 200 and all(x <= y for x, y in zip(b, b[1:]))
    shares = [int(rp[b[i + 1]] - rp[b[i]]) for i in range(parts)]
    assert max(shares) - min(shares) <= 2 * counts.max() + 1
