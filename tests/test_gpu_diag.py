"""The L2 -> SM gather probe (kairo_gather_probe): argument checks and a
plausible rate on an L2-resident buffer."""

from __future__ import annotations

import ctypes

import pytest
import torch

from kairo_b200 import _lib

pytestmark = pytest.mark.gpu


def _probe(buf, nbytes, load, iters=50):
    out = ctypes.c_double(0.0)
    st = _lib.lib().kairo_gather_probe(buf.data_ptr(), nbytes, load, iters, ctypes.byref(out),
                                       _lib.stream_handle(buf.device))
    return st, out.value


def test_gather_probe_rate():
    buf = torch.zeros(32 << 20, dtype=torch.uint8, device="cuda")
    for load in (2048, 16384):
        st, gbs = _probe(buf, buf.numel(), load)
        assert st == 0
        assert 100.0 < gbs < 200000.0


def test_gather_probe_rejects_bad_arguments():
    buf = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    invalid = _lib.INVALID_VALUE
    assert _probe(buf, buf.numel(), 1000)[0] == invalid       # not a multiple of 16
    assert _probe(buf, buf.numel(), 3 * 4096)[0] == invalid   # does not divide the 32 KiB stage
    assert _probe(buf, 1024, 4096)[0] == invalid              # buffer smaller than one copy
    assert _probe(buf, buf.numel(), 4096, iters=0)[0] == invalid
