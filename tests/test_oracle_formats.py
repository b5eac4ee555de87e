"""The CPU oracle against golden vectors (gguf-py) and the reference's own
known-answer semantics for block decode and activation quantization."""
from pathlib import Path

import numpy as np
import pytest

import oracle
from inferq_b200 import quants as Q

G = np.load(Path(__file__).parent / "golden" / "formats.npz")


@pytest.mark.parametrize("dt", [Q.Q4_K, Q.Q5_K, Q.Q6_K, Q.Q8_0])
def test_block_decode_is_bit_exact_against_gguf_py(dt):
    name = Q.NAMES[dt]
    blocks, ref = G[f"{name}_bytes"], G[f"{name}_f32"]
    got = oracle.dequant(dt, blocks, *ref.shape)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_q8_0_activation_quantization_matches_gguf_py():
    got = oracle.quant_q80(G["act_f32"])
    assert np.array_equal(got, G["act_q8_0"].ravel())


def test_q8k_quantization_follows_candle_from_float():
    # iscale = -128/max of the largest-magnitude value; that value maps to -128.
    x = np.linspace(-1.0, 0.5, 256, dtype=np.float32)
    blk = oracle.quant_q8k(x)
    d = blk[:4].view(np.float32)[0]
    qs = blk[4:260].view(np.int8)
    bs = blk[260:292].view(np.int16)
    assert qs[0] == -128 * np.sign(x[0]) * -1 or qs[0] == -128
    assert d == np.float32(1.0) / (np.float32(-128.0) / np.float32(-1.0))
    assert np.array_equal(bs, qs.astype(np.int32).reshape(16, 16).sum(1).astype(np.int16))
    # first occurrence wins on equal magnitude: +1 before -1 gives d < 0
    y = np.zeros(256, np.float32)
    y[3], y[9] = 1.0, -1.0
    blk = oracle.quant_q8k(y)
    assert blk[:4].view(np.float32)[0] < 0 and blk[4 + 3].view(np.int8) == -128
    assert blk[4 + 9].view(np.int8) == 127  # +128 capped at 127
    # an all-zero block
    z = oracle.quant_q8k(np.zeros(256, np.float32))
    assert not z.any()


@pytest.mark.parametrize("dt,cols", [(Q.Q4_K, 512), (Q.Q5_K, 512), (Q.Q6_K, 768), (Q.Q8_0, 256)])
def test_reference_and_device_orders_agree_to_f32_rounding(dt, cols):
    import torch
    torch.manual_seed(dt)
    w = Q.encode(torch.randn(24, cols) * 0.02, dt).numpy()
    x = np.random.default_rng(dt).standard_normal((3, cols)).astype(np.float32)
    a = oracle.qmatvec(dt, w, 24, cols, x, order=0)
    b = oracle.qmatvec(dt, w, 24, cols, x, order=1, ksplit=2 if dt != Q.Q8_0 else 1)
    deq = oracle.dequant(dt, w, 24, cols)
    exact = x.astype(np.float64) @ deq.astype(np.float64).T
    scale = np.abs(x).max() * np.abs(deq).sum(1).max()
    assert np.abs(a - b).max() <= 1e-5 * scale
    # the reference's own tolerance vs f32 matmul of the dequantized matrix
    # (src/gguf.rs:1741-1775 direct_matrix_matches_its_dequantized_reference)
    assert np.abs(a - exact).max() < 2e-2


def test_argmax_takes_the_last_max_and_skips_non_finite():
    assert oracle.argmax(np.array([1, 3, 3, 2], np.float32)) == 2
    assert oracle.argmax(np.array([np.nan, 1, np.inf, -np.inf], np.float32)) == 1
    assert oracle.argmax(np.array([np.nan], np.float32)) == -1


@pytest.mark.parametrize("dtype", [12, 13, 14, 8])
def test_avx2_reference_order_equals_the_scalar_restatement(dtype):
    """The oracle's AVX2 reference-order kernels (the CPU baseline's fast
    path) are bitwise its scalar restatement of src/qgemm.rs, for 1..11
    input rows (several 8-row tiles)."""
    import torch
    from inferq_b200 import quants as Q
    if not oracle.have_avx2():
        pytest.skip("no AVX2 on this CPU")
    rows, cols = 37, 1024
    w = Q.encode(torch.randn(rows, cols, generator=torch.Generator().manual_seed(dtype)) * 0.02, dtype).numpy()
    for k in (1, 4, 8, 11):
        x = np.random.default_rng(k).standard_normal((k, cols)).astype(np.float32)
        fast = oracle.qmatvec(dtype, w, rows, cols, x)
        oracle.force_scalar(True)
        try:
            slow = oracle.qmatvec(dtype, w, rows, cols, x)
        finally:
            oracle.force_scalar(False)
        assert np.array_equal(fast.view(np.uint32), slow.view(np.uint32)), k


@pytest.mark.parametrize("nh,nkv,hd,positions", [(16, 2, 256, 700), (8, 2, 72, 33), (4, 4, 64, 1)])
def test_avx2_attention_scan_equals_the_scalar_restatement(nh, nkv, hd, positions):
    """The oracle's AVX2 attention loops (dot8's eight lanes as one vector,
    the value sum eight output elements at a time) are bitwise its scalar
    restatement of src/qwen/quantized_attention.rs:155-178."""
    if not oracle.have_avx2():
        pytest.skip("no AVX2 on this CPU")
    rng = np.random.default_rng(positions)
    q = rng.standard_normal((nh, hd)).astype(np.float32)
    gate = rng.standard_normal((nh, hd)).astype(np.float32)
    keys = (3 * rng.standard_normal((positions, nkv, hd))).astype(np.float32)
    values = rng.standard_normal((positions, nkv, hd)).astype(np.float32)
    fast = oracle.attend(q, gate, keys, values, nh, nkv, hd)
    oracle.force_scalar(True)
    try:
        slow = oracle.attend(q, gate, keys, values, nh, nkv, hd)
    finally:
        oracle.force_scalar(False)
    assert np.array_equal(fast.view(np.uint32), slow.view(np.uint32))
