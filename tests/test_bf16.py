"""BF16 matrices (QuantizedMatrix accepts BF16, src/gguf.rs:305-316) and BF16
1-D tensors (loaded as f32, src/gguf.rs:1487-1495): the oracle on the CPU,
the device operator against the oracle, the model loader's widening."""
import numpy as np
import pytest
import torch

import oracle
from inferq_b200 import quants as Q


def _bf16(rows, cols, seed):
    x = torch.randn(rows, cols, generator=torch.Generator().manual_seed(seed)) * 0.05
    return Q.encode(x, Q.BF16).numpy()


def test_oracle_bf16_decode_and_product():
    """Decode is the exact widening; the product multiplies input rows
    rounded to bf16 and sums exact products (checked against float64)."""
    w = _bf16(9, 64, 1)
    ref = torch.from_numpy(w.copy()).view(torch.bfloat16).float().numpy()
    assert np.array_equal(oracle.dequant(Q.BF16, w, 9, 64), ref)
    x = np.random.default_rng(2).standard_normal((3, 64)).astype(np.float32)
    xb = torch.from_numpy(x).to(torch.bfloat16).float().numpy().astype(np.float64)
    y = oracle.qmatvec(Q.BF16, w, 9, 64, x)
    want = xb @ ref.astype(np.float64).T
    assert np.all(np.abs(y - want) <= 1e-6 * (np.abs(xb) @ np.abs(ref.astype(np.float64)).T) + 1e-9)


@pytest.mark.gpu
def test_device_bf16_matrix_matches_the_oracle(cuda):
    from inferq_b200 import _lib
    rows, cols = 300, 1024
    w = _bf16(rows, cols, 3)
    m = _lib.Matrix(Q.BF16, w, rows, cols)
    assert np.array_equal(m.dequantize(), oracle.dequant(Q.BF16, w, rows, cols))
    for k in (1, 4, 8, 11):
        x = np.random.default_rng(k).standard_normal((k, cols)).astype(np.float32)
        y = m.forward_rows(x)
        ref = oracle.qmatvec(Q.BF16, w, rows, cols, x)
        # the same exact products, summed in another order: within 1e-5 of their magnitudes
        xb = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
        bound = 1e-5 * (np.abs(xb) @ np.abs(oracle.dequant(Q.BF16, w, rows, cols)).T) + 1e-7
        assert np.all(np.abs(y - ref) <= bound), k
    with pytest.raises(_lib.IqError):
        m.forward_wide(torch.zeros(64, cols, device="cuda"))


@pytest.mark.gpu
def test_model_takes_bf16_vectors(cuda):
    """A checkpoint whose norm weights are BF16 runs exactly like the same
    checkpoint with those weights widened to F32."""
    from inferq_b200 import synth
    from inferq_b200.model import Model, State
    cfg = synth.tiny()
    t32, tbf = [], []
    for t in synth.generate(cfg, seed=8):
        if t.dtype == Q.F32 and "norm" in t.name:
            b = t.data.to(torch.bfloat16)
            tbf.append(synth.Tensor(t.name, Q.BF16, t.shape, b.view(torch.uint8)))
            t32.append(synth.Tensor(t.name, Q.F32, t.shape, b.float()))
        else:
            t32.append(t)
            tbf.append(t)
    a = State(Model(cfg, t32), 32).forward([5, 6, 7], logits=True)[1]
    b = State(Model(cfg, tbf), 32).forward([5, 6, 7], logits=True)[1]
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
