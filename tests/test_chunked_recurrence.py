"""The wide pass's chunked (WY) DeltaNet recurrence against the sequential
delta rule, on the CPU oracle.

The device's chunked kernels are held bitwise to the oracle's restatement of
the chunked form (tests/test_wide_pass_gpu.py); this file checks the algebra
of that form itself: over a chunk of rows it must give the outputs and the
state of the sequential rule (src/qwen/deltanet.rs:170-217, whose own known
answers tests/test_known_answers.py holds) up to f32 rounding order,
including decays strong enough that a product of per-row decays would
underflow (the form only uses exp of differences of cumulative log-decays).
"""
import numpy as np
import pytest

import oracle

f32 = np.float32


def _rows(rng, C, dk, dv, lg_lo, lg_hi):
    q = rng.standard_normal((C, dk)).astype(f32)
    k = rng.standard_normal((C, dk)).astype(f32)
    q /= np.sqrt((q * q).sum(axis=1, keepdims=True) + 1e-6).astype(f32)
    k /= np.sqrt((k * k).sum(axis=1, keepdims=True) + 1e-6).astype(f32)
    v = rng.standard_normal((C, dv)).astype(f32)
    beta = rng.uniform(0.05, 0.95, C).astype(f32)
    lg = rng.uniform(lg_lo, lg_hi, C).astype(f32)
    S0 = (0.1 * rng.standard_normal((dk, dv))).astype(f32)
    return q, k, v, beta, lg, S0


def _sequential(q, k, v, beta, lg, S0):
    C, dk = q.shape
    dv = v.shape[1]
    S = S0.reshape(-1).copy()
    out = np.empty((C, dv), f32)
    for t in range(C):
        o, S = oracle.delta_step(q[t], k[t], v[t], [lg[t]], [beta[t]], 1, dk, dv, S)
        out[t] = o
    return out, S.reshape(dk, dv)


@pytest.mark.parametrize("dk,dv", [(64, 64), (128, 128), (128, 32)])
@pytest.mark.parametrize("C", [1, 5, 32])
@pytest.mark.parametrize("decay", ["moderate", "strong", "none"])
def test_chunked_form_equals_the_sequential_rule(dk, dv, C, decay):
    lo, hi = {"moderate": (-0.5, -0.01), "strong": (-12.0, -8.0), "none": (0.0, 0.0)}[decay]
    rng = np.random.default_rng(dk * 1000 + dv * 10 + C)
    q, k, v, beta, lg, S0 = _rows(rng, C, dk, dv, lo, hi)
    ref_o, ref_S = _sequential(q, k, v, beta, lg, S0)
    o, S = oracle.delta_chunk(q, k, v, beta, lg, S0)
    assert np.isfinite(o).all() and np.isfinite(S).all()
    scale_o = max(1.0, float(np.abs(ref_o).max()))
    scale_S = max(1.0, float(np.abs(ref_S).max()))
    assert np.abs(o - ref_o).max() <= 2e-6 * scale_o, (decay, np.abs(o - ref_o).max())
    assert np.abs(S - ref_S).max() <= 2e-6 * scale_S, (decay, np.abs(S - ref_S).max())


def test_chunks_chain_like_one_sequence():
    """Two consecutive chunks (the second starting from the first's state)
    equal 48 sequential rows."""
    rng = np.random.default_rng(11)
    q, k, v, beta, lg, S0 = _rows(rng, 48, 128, 64, -0.3, -0.01)
    ref_o, ref_S = _sequential(q, k, v, beta, lg, S0)
    o1, S1 = oracle.delta_chunk(q[:32], k[:32], v[:32], beta[:32], lg[:32], S0)
    o2, S2 = oracle.delta_chunk(q[32:], k[32:], v[32:], beta[32:], lg[32:], S1)
    o = np.concatenate([o1, o2])
    assert np.abs(o - ref_o).max() <= 2e-6 * max(1.0, float(np.abs(ref_o).max()))
    assert np.abs(S2 - ref_S).max() <= 2e-6 * max(1.0, float(np.abs(ref_S).max()))
