"""The skinny quantized GEMV on the GPU against the CPU oracle.

Bit-exact where the arithmetic is defined identically (block decode; the
device accumulation order restated by the oracle), within f32 rounding of the
reference's AVX2 lane order, and independent of how many rows run together.
"""
import numpy as np
import pytest
import torch

import oracle
from inferq_b200 import _lib
from inferq_b200 import quants as Q

pytestmark = pytest.mark.gpu

SHAPES = [
    (Q.Q4_K, 40, 512), (Q.Q4_K, 1024, 2048), (Q.Q5_K, 48, 768), (Q.Q6_K, 37, 512),
    (Q.Q6_K, 2048, 512), (Q.Q6_K, 96, 2048), (Q.Q8_0, 33, 256), (Q.Q8_0, 2048, 4096),
    (Q.F32, 64, 2048),
]


def _weights(dt, rows, cols, seed):
    g = torch.Generator().manual_seed(seed)
    return Q.encode(torch.randn(rows, cols, generator=g) * 0.02, dt).numpy()


@pytest.mark.parametrize("dt,rows,cols", SHAPES)
def test_device_decode_is_bit_exact(cuda, dt, rows, cols):
    w = _weights(dt, rows, cols, 1)
    m = _lib.Matrix(dt, w, rows, cols)
    got = m.dequantize()
    ref = oracle.dequant(dt, w, rows, cols)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    ids = np.array([rows - 1, 0, rows // 2], np.int32)
    assert np.array_equal(m.dequantize(ids), ref[ids])


@pytest.mark.parametrize("dt,rows,cols", SHAPES)
@pytest.mark.parametrize("k", [1, 3, 8, 11])
def test_gemv_matches_oracle(cuda, dt, rows, cols, k):
    w = _weights(dt, rows, cols, 2)
    x = np.random.default_rng(k).standard_normal((k, cols)).astype(np.float32)
    x[0] *= 30.0
    m = _lib.Matrix(dt, w, rows, cols)
    got = m.forward_rows(x)
    if dt == Q.F32:
        ref = x.astype(np.float64) @ w.view(np.float32).reshape(rows, cols).astype(np.float64).T
        assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max()
        return
    dev = oracle.qmatvec(dt, w, rows, cols, x, order=1, ksplit=_lib.ksplit(dt, rows, cols))
    assert np.array_equal(got.view(np.uint32), dev.view(np.uint32)), np.abs(got - dev).max()
    ref = oracle.qmatvec(dt, w, rows, cols, x, order=0)
    scale = np.abs(x).max(1, keepdims=True) * np.abs(oracle.dequant(dt, w, rows, cols)).sum(1)[None, :]
    assert (np.abs(got - ref) <= 1e-5 * scale).all()


@pytest.mark.parametrize("dt,rows,cols", [s for s in SHAPES if s[0] != Q.F32])
def test_a_row_does_not_depend_on_the_rows_beside_it(cuda, dt, rows, cols):
    w = _weights(dt, rows, cols, 3)
    x = np.random.default_rng(5).standard_normal((8, cols)).astype(np.float32)
    m = _lib.Matrix(dt, w, rows, cols)
    together = m.forward_rows(x)
    for i in range(8):
        alone = m.forward_rows(x[i:i + 1])
        assert np.array_equal(alone[0].view(np.uint32), together[i].view(np.uint32))


def test_leading_rows_is_a_prefix(cuda):
    w = _weights(Q.Q6_K, 300, 512, 4)
    m = _lib.Matrix(Q.Q6_K, w, 300, 512)
    head = m.leading_rows(128)
    x = np.random.default_rng(1).standard_normal((2, 512)).astype(np.float32)
    assert np.array_equal(head.forward_rows(x), m.forward_rows(x)[:, :128])


def test_device_resident_weights_upload(cuda):
    t = Q.encode(torch.randn(64, 512, device="cuda") * 0.02, Q.Q4_K)
    m = _lib.Matrix(Q.Q4_K, t, 64, 512)
    assert np.array_equal(m.dequantize(), oracle.dequant(Q.Q4_K, t.cpu().numpy(), 64, 512))
