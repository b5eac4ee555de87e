"""The GEMV entry point that allocates no device memory.

iq_matrix_forward_device_noalloc serves callers that must not allocate while
they run (a host that partitions device memory up front for its own pool, or
a decode thread that cannot absorb cudaMalloc's implicit synchronization).
It keeps its scratch in a fixed array inside the library.  Here it must give
exactly what the allocating entry point gives, on two calls in a row (the
second call reuses the array the first one left behind), and it must refuse
requests larger than that array.  This file runs last so a failure here
cannot hide failures elsewhere.
"""
import ctypes

import numpy as np
import pytest
import torch

from inferq_b200 import _lib
from inferq_b200 import quants as Q

pytestmark = pytest.mark.gpu

SHAPES = [(Q.Q4_K, 1024, 2048), (Q.Q6_K, 300, 4096), (Q.Q8_0, 2048, 4096), (Q.Q5_K, 64, 512), (Q.F32, 65, 2048)]


def _bits(t):
    return t.cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("dt,rows,cols", SHAPES)
def test_noalloc_forward_matches_the_allocating_forward(cuda, dt, rows, cols):
    L = _lib.lib()
    g = torch.Generator(device="cuda").manual_seed(dt)
    w = Q.encode(torch.randn(rows, cols, device="cuda", generator=g) * 0.02, dt)
    m = _lib.Matrix(dt, w, rows, cols)
    for k in (8, 3):  # two calls in a row with different row counts
        x = torch.randn(k, cols, device="cuda", generator=g)
        want = torch.empty(k, rows, device="cuda")
        got = torch.full((k, rows), float("nan"), device="cuda")
        _lib.check(L.iq_matrix_forward_device(m._h, x.data_ptr(), k, want.data_ptr(), None))
        _lib.check(L.iq_matrix_forward_device_noalloc(m._h, x.data_ptr(), k, got.data_ptr(), None))
        torch.cuda.synchronize()
        assert np.array_equal(_bits(got), _bits(want))


def test_noalloc_forward_rejects_requests_beyond_its_scratch(cuda):
    L = _lib.lib()
    w = Q.encode(torch.randn(16, 8192, device="cuda") * 0.02, Q.Q4_K)
    m = _lib.Matrix(Q.Q4_K, w, 16, 8192)
    x = torch.randn(1, 8192, device="cuda")
    y = torch.empty(1, 16, device="cuda")
    assert L.iq_matrix_forward_device_noalloc(m._h, x.data_ptr(), 1, y.data_ptr(), None) == -1
    assert b"at most 4096 columns" in L.iq_last_error()
    w2 = Q.encode(torch.randn(16, 512, device="cuda") * 0.02, Q.Q4_K)
    m2 = _lib.Matrix(Q.Q4_K, w2, 16, 512)
    x2 = torch.randn(9, 512, device="cuda")
    y2 = torch.empty(9, 16, device="cuda")
    assert L.iq_matrix_forward_device_noalloc(m2._h, x2.data_ptr(), 9, y2.data_ptr(), None) == -1
    assert b"1..8 input rows" in L.iq_last_error()
