"""The wide Q8_0 product on the tensor cores (iq_matrix_forward_wide) against
the CPU oracle.

The reference computes prefill through the same QuantizedMatrix::forward as
decode (src/runtime.rs:748-771, src/gguf.rs:406-456), so the wide product has
to give the integer block dots of src/qgemm.rs:369-397 (Q8_0 x Q8_0).  Its f32
order is one FMA per block in ascending block order: bitwise the oracle's
device order with one K chunk (oracle/iq_oracle_dot.c dev_block_chunks).
"""
import os

import numpy as np
import pytest
import torch

import oracle
from inferq_b200 import _lib
from inferq_b200 import quants as Q

pytestmark = pytest.mark.gpu


def _weights(rows, cols, seed):
    g = torch.Generator().manual_seed(seed)
    return Q.encode(torch.randn(rows, cols, generator=g) * 0.02, Q.Q8_0).numpy()


def _inputs(n, cols, seed):
    x = np.random.default_rng(seed).standard_normal((n, cols)).astype(np.float32)
    x[0] *= 30.0
    if n > 2:
        x[2] = 0.0          # an all-zero row (block scale 0)
        x[1, :64] = 1e-30   # tiny blocks
    return x


@pytest.mark.parametrize("rows,cols,n", [
    (128, 128, 1), (200, 1024, 37), (128, 512, 128), (300, 256, 129), (1000, 2048, 300),
])
def test_wide_matches_the_oracle_bitwise(cuda, rows, cols, n):
    w = _weights(rows, cols, rows + n)
    x = _inputs(n, cols, n)
    m = _lib.Matrix(Q.Q8_0, w, rows, cols)
    got = m.forward_wide(torch.from_numpy(x).cuda()).cpu().numpy()
    ref = oracle.qmatvec(Q.Q8_0, w, rows, cols, x, order=1, ksplit=1)
    bad = np.argwhere(got.view(np.uint32) != ref.view(np.uint32))
    assert len(bad) == 0, (len(bad), bad[:5], np.abs(got - ref).max())


def test_wide_equals_the_narrow_path_where_it_runs_unsplit(cuda):
    rows, cols = 16384, 128
    assert _lib.ksplit(Q.Q8_0, rows, cols) == 1
    w = _weights(rows, cols, 7)
    x = _inputs(24, cols, 3)
    m = _lib.Matrix(Q.Q8_0, w, rows, cols)
    wide = m.forward_wide(torch.from_numpy(x).cuda()).cpu().numpy()
    narrow = m.forward_rows(x)
    assert np.array_equal(wide.view(np.uint32), narrow.view(np.uint32))
    # and at a split shape, equal to the oracle's one-chunk order instead
    rows, cols = 512, 2048
    assert _lib.ksplit(Q.Q8_0, rows, cols) > 1
    w = _weights(rows, cols, 8)
    m = _lib.Matrix(Q.Q8_0, w, rows, cols)
    wide = m.forward_wide(torch.from_numpy(x[:5]).cuda().repeat(1, 16)).cpu().numpy()
    ref = oracle.qmatvec(Q.Q8_0, w, rows, cols, np.tile(x[:5], (1, 16)), order=1, ksplit=1)
    assert np.array_equal(wide.view(np.uint32), ref.view(np.uint32))


def test_wide_rows_do_not_depend_on_their_neighbours_at_full_width(cuda):
    """512 input rows at a 35B projection shape: each output row equals the
    same input row run alone (size-independent property), and the result is
    within f32 rounding of a float64 product of the decoded operands."""
    rows, cols, n = 8192, 2048, 512
    g = torch.Generator(device="cuda").manual_seed(11)
    w = Q.encode(torch.randn(rows, cols, device="cuda", generator=g) * 0.02, Q.Q8_0)
    m = _lib.Matrix(Q.Q8_0, w, rows, cols)
    x = torch.randn(n, cols, device="cuda", generator=g)
    y = m.forward_wide(x)
    for i in (0, 1, 127, 128, 300, 511):
        yi = m.forward_wide(x[i:i + 1])
        assert torch.equal(yi[0].view(torch.int32), y[i].view(torch.int32)), i
    # float64 reference over the quantized operands, sampled rows
    ids = torch.tensor([0, 1, 2, 4095, 8191])
    wd = torch.from_numpy(m.dequantize(ids.numpy().astype(np.int32))).double()
    xq = torch.from_numpy(oracle.dequant(Q.Q8_0, oracle.quant_q80(x.cpu().numpy()), n, cols)).double()
    ref = xq @ wd.T
    err = (y[:, ids].cpu().double() - ref).abs().max().item()
    assert err <= 1e-4 * ref.abs().max().item(), err


@pytest.mark.parametrize("rows,cols,n", [
    (128, 256, 1), (200, 512, 37), (128, 1024, 64), (300, 256, 129), (1000, 2048, 300),
])
@pytest.mark.parametrize("dt", [Q.Q4_K, Q.Q6_K])
def test_wide_kquant_matches_the_oracle_bitwise(cuda, dt, rows, cols, n):
    """K-quants x Q8_K: scale-folded f16 operands (Q4_K: sc*q with split
    half-block accumulators and the min term; Q6_K: the scale split into
    16*sh + sl, two accumulators) on the tensor cores, bitwise the one-chunk
    order."""
    g = torch.Generator().manual_seed(rows + 7 * n)
    w = Q.encode(torch.randn(rows, cols, generator=g) * 0.02, dt).numpy()
    x = _inputs(n, cols, n + 1)
    m = _lib.Matrix(dt, w, rows, cols)
    got = m.forward_wide(torch.from_numpy(x).cuda()).cpu().numpy()
    ref = oracle.qmatvec(dt, w, rows, cols, x, order=1, ksplit=1)
    bad = np.argwhere(got.view(np.uint32) != ref.view(np.uint32))
    assert len(bad) == 0, (len(bad), bad[:5], np.abs(got - ref).max())


@pytest.mark.parametrize("dt", [Q.Q4_K, Q.Q6_K])
def test_wide_kquant_at_full_width_equals_rows_run_alone(cuda, dt):
    rows, cols, n = 4096, 2048, 512
    g = torch.Generator(device="cuda").manual_seed(12)
    w = Q.encode(torch.randn(rows, cols, device="cuda", generator=g) * 0.02, dt)
    m = _lib.Matrix(dt, w, rows, cols)
    x = torch.randn(n, cols, device="cuda", generator=g)
    y = m.forward_wide(x)
    for i in (0, 63, 64, 511):
        assert torch.equal(m.forward_wide(x[i:i + 1])[0].view(torch.int32), y[i].view(torch.int32)), i


Q5K = pytest.mark.skipif(not os.environ.get("IQ_WIDE_Q5K"),
                         reason="the Q5_K wide product is enabled by IQ_WIDE_Q5K")


def _q5k_extreme(rows, q):
    """Q5_K rows whose every scale is 63, every min 0, every quant q, d = 1."""
    blk = np.zeros(176, np.uint8)
    blk[0:2] = np.frombuffer(np.float16(1.0).tobytes(), np.uint8)
    blk[4:8] = 0xFF            # sc0-3 = 63, top bits of sc4-7 = 3
    blk[12:16] = 0x0F          # sc4-7 low nibbles 15, mins 0
    blk[16:48] = 0xFF if q & 16 else 0
    blk[48:176] = (q & 15) * 0x11
    return np.tile(blk, rows * 2)  # two blocks per row (512 columns)


@Q5K
@pytest.mark.parametrize("rows,cols,n", [
    (128, 256, 1), (200, 512, 37), (128, 1024, 64), (300, 256, 129), (1000, 2048, 300),
])
def test_wide_q5k_matches_the_oracle_bitwise(cuda, rows, cols, n):
    """Q5_K x Q8_K: the centred operand sc*(q-16) in half-block
    accumulators, the centring term 16*sum sc*bsum from one more MMA, the
    integers summed exactly: bitwise the one-chunk order."""
    g = torch.Generator().manual_seed(rows + 5 * n)
    w = Q.encode(torch.randn(rows, cols, generator=g) * 0.02, Q.Q5_K).numpy()
    x = _inputs(n, cols, n + 2)
    m = _lib.Matrix(Q.Q5_K, w, rows, cols)
    got = m.forward_wide(torch.from_numpy(x).cuda()).cpu().numpy()
    ref = oracle.qmatvec(Q.Q5_K, w, rows, cols, x, order=1, ksplit=1)
    bad = np.argwhere(got.view(np.uint32) != ref.view(np.uint32))
    assert len(bad) == 0, (len(bad), bad[:5], np.abs(got - ref).max())


@Q5K
@pytest.mark.parametrize("q", [0, 31, 16])
def test_wide_q5k_is_exact_at_its_magnitude_bound(cuda, q):
    """Every scale 63 and inputs of one sign (every Q8_K quant -128): each
    half-block accumulator reaches 128 * 63 * 16 * 128, just below 2^24, and
    the centring term 16 * 8 * 63 * 4096 exceeds it (q = 0: the exact block
    sum is 0, which any rounding inside the accumulation would miss)."""
    rows, cols = 128, 512
    w = _q5k_extreme(rows, q)
    x = np.ones((3, cols), np.float32)
    x[1] *= -1.0
    m = _lib.Matrix(Q.Q5_K, w, rows, cols)
    got = m.forward_wide(torch.from_numpy(x).cuda()).cpu().numpy()
    ref = oracle.qmatvec(Q.Q5_K, w, rows, cols, x, order=1, ksplit=1)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), (got[:, :2], ref[:, :2])
    if q == 0:
        assert not ref.any()


def test_wide_rejects_what_it_does_not_support(cuda):
    w = Q.encode(torch.randn(64, 256) * 0.02, Q.Q5_K).numpy()
    m = _lib.Matrix(Q.Q5_K, w, 64, 256)
    if not os.environ.get("IQ_WIDE_Q5K"):
        with pytest.raises(_lib.IqError):
            m.forward_wide(torch.zeros(4, 256, device="cuda"))
    w8 = _weights(64, 128, 1)
    m8 = _lib.Matrix(Q.Q8_0, w8, 64, 128)
    with pytest.raises(_lib.IqError):  # no input rows
        m8.forward_wide(torch.zeros(0, 128, device="cuda"))
