"""The exactness argument behind the wide (tensor-core) products, checked
exhaustively over the formats' value ranges on the CPU.

The wide kernels form integer block dots as f16 x f16 -> f32 MMAs.  That is
exact only if every operand value is an f16 integer and every partial sum of
a TMEM accumulator stays below 2^24; the recombinations must round the exact
integer once, as (float)isum does in the reference (src/qgemm.rs
accumulates isum as i32 and converts once).  These tests pin each claim the
kernels rely on (inferq_b200/csrc/wide.cu).
"""
import numpy as np

F24 = 1 << 24


def _f16_exact(values):
    v = np.asarray(values, dtype=np.int64)
    return np.array_equal(v.astype(np.float16).astype(np.int64), v)


def test_q8_0_operands_and_block_sums_are_exact():
    assert _f16_exact(np.arange(-128, 128))  # weight quants and Q8_0 input quants
    assert 32 * 128 * 128 < F24               # one block's sum in a fresh accumulator


def test_q4k_scale_folded_operand_and_half_block_sums_are_exact():
    sc, q = np.meshgrid(np.arange(64), np.arange(16))
    assert _f16_exact(sc * q)                 # A = sc * q <= 945
    assert _f16_exact(np.arange(-128, 128))   # Q8_K input quants
    half = 128 * 945 * 128
    assert half < F24                         # each half-block accumulator
    assert 2 * half >= F24                    # ... which is why the block is split


def test_q4k_half_sums_recombine_like_the_integer_conversion():
    """a + b in f32 (a, b exact integers) rounds the exact sum once, the same
    as converting the i32 sum: checked on sums straddling 2^24..2^25."""
    rng = np.random.default_rng(0)
    a = rng.integers(-15_482_880, 15_482_881, 200_000)
    b = rng.integers(-15_482_880, 15_482_881, 200_000)
    a[:1000] = 15_482_880
    b[:1000] = rng.integers(1_000_000, 15_482_881, 1000)
    got = (a.astype(np.float32) + b.astype(np.float32)).astype(np.float32)
    ref = (a + b).astype(np.float32)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_q4k_min_term_operands_are_exact():
    mn = np.arange(64)
    assert _f16_exact(mn) and _f16_exact(64 * mn)
    bsum = np.arange(-32 * 128, 32 * 127 + 1)  # 32-element sums of Q8_K quants
    lo = bsum & 63
    hi = (bsum - lo) // 64
    assert np.array_equal(64 * hi + lo, bsum)
    assert lo.min() >= 0 and lo.max() < 64 and hi.min() >= -64 and hi.max() < 64
    assert _f16_exact(lo) and _f16_exact(hi)
    assert 8 * 63 * 63 + 8 * (64 * 63) * 64 < F24  # the min accumulator


def test_q6k_scale_split_is_exact_and_recombines_once():
    sc = np.arange(-128, 128)
    sh, sl = sc >> 4, sc & 15
    assert np.array_equal(16 * sh + sl, sc)
    v = np.arange(-32, 32)                     # q - 32
    assert _f16_exact(np.outer(sl, v)) and _f16_exact(np.outer(sh, v))
    assert not _f16_exact(np.outer(sc, v))     # why the split is needed
    assert 256 * 15 * 32 * 128 < F24 and 256 * 8 * 32 * 128 < F24
    # fmaf(16, hi, lo) == (float)(16*hi + lo): one rounding of the exact value
    rng = np.random.default_rng(1)
    hi = rng.integers(-8_388_608, 8_388_609, 200_000)
    lo = rng.integers(-15_728_640, 15_728_641, 200_000)
    exact = 16 * hi + lo
    ref = exact.astype(np.float32)
    fma = (16.0 * hi.astype(np.float64) + lo.astype(np.float64)).astype(np.float32)  # f64 holds it exactly
    assert np.array_equal(fma.view(np.uint32), ref.view(np.uint32))


def test_q5k_centred_operand_and_centring_term_are_exact():
    """Q5_K: sc * q (q <= 31) reaches 1953 and a half block would pass 2^24,
    so the operand is centred, A = sc * (q - 16); the centring term
    c = sum_s sc[s] * bsum_s comes from (sc, 64 sc) x (bsum mod 64,
    bsum div 64) and isum = a + b + 16 c as exact int32."""
    sc, q = np.meshgrid(np.arange(64), np.arange(32))
    assert _f16_exact(sc * q) and 128 * 1953 * 128 >= F24   # why it is centred
    assert _f16_exact(sc * (q - 16))
    assert 128 * 63 * 16 * 128 < F24                        # each half block
    s = np.arange(64)
    assert _f16_exact(s) and _f16_exact(64 * s)
    assert 8 * 63 * 63 + 8 * (64 * 63) * 64 < F24            # the c accumulator
    assert 256 * 63 * 31 * 128 < 2 ** 31                     # isum fits int32
    # the decomposition itself, on random and on extreme blocks
    rng = np.random.default_rng(2)
    for trial in range(200):
        if trial < 4:
            qv = np.full(256, (0, 31, 16, 15)[trial])
            scv = np.full(8, 63)
            x = np.full(256, -128)
        else:
            qv = rng.integers(0, 32, 256)
            scv = rng.integers(0, 64, 8)
            x = rng.integers(-128, 128, 256)
        a_op = np.repeat(scv, 32) * (qv - 16)
        a, b = int((a_op[:128] * x[:128]).sum()), int((a_op[128:] * x[128:]).sum())
        assert abs(a) < F24 and abs(b) < F24
        bsum = x.reshape(8, 32).sum(axis=1)
        lo = bsum & 63
        hi = (bsum - lo) // 64
        c = int((scv * lo).sum() + (64 * scv * hi).sum())
        assert a + b + 16 * c == int((np.repeat(scv, 32) * qv * x).sum())
