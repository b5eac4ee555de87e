"""The reference's own known-answer tests for the layer math, applied to the
CPU oracle (and, where the library has host logic, to libiq).  Each test
cites the reference test it restates; inputs and expected values are the
reference test's own.  No GPU is needed.
"""
import ctypes

import numpy as np
import pytest

import oracle
from inferq_b200 import _lib

f32 = np.float32


def test_delta_rule_updates_and_reuses_state():
    """src/qwen/deltanet.rs:415-449: one head, key/value dim 2, g 0, beta 1;
    two steps with the same inputs both give v / sqrt(2)."""
    state = np.zeros(4, f32)
    for _ in range(2):
        out, state = oracle.delta_step([1, 0], [1, 0], [2, 3], [0], [1], 1, 2, 2, state)
        assert abs(out[0] - 2 / np.sqrt(f32(2))) < 1e-6
        assert abs(out[1] - 3 / np.sqrt(f32(2))) < 1e-6


def _strided_reference(q, k, v, g, beta, heads, kd, vd, state):
    """strided_recurrence_reference (deltanet.rs:373-412), column by column,
    in float32 with every product rounded."""
    state = state.copy()
    out = np.zeros(heads * vd, f32)
    qs = f32(1) / np.sqrt(f32(kd))
    for h in range(heads):
        sb, qb, vb = h * kd * vd, h * kd, h * vd
        decay = np.exp(f32(g[h]), dtype=f32)
        state[sb:sb + kd * vd] *= decay
        for j in range(vd):
            pred = f32(0)
            for i in range(kd):
                pred = f32(pred + f32(state[sb + i * vd + j] * k[qb + i]))
            delta = f32(f32(v[vb + j] - pred) * f32(beta[h]))
            for i in range(kd):
                state[sb + i * vd + j] = f32(state[sb + i * vd + j] + f32(k[qb + i] * delta))
        for j in range(vd):
            val = f32(0)
            for i in range(kd):
                val = f32(val + f32(f32(state[sb + i * vd + j] * q[qb + i]) * qs))
            out[vb + j] = val
    return out, state


def test_contiguous_recurrence_matches_strided_reference():
    """deltanet.rs:451-502: heads 2, key dim 4, value dim 3, the reference's
    ramps for q, k, v and the initial state; agreement within 1e-6."""
    heads, kd, vd = 2, 4, 3
    q = np.array([(i - 3.0) / 7.0 for i in range(heads * kd)], f32)
    k = np.array([(5.0 - i) / 9.0 for i in range(heads * kd)], f32)
    v = np.array([(i + 1.0) / 5.0 for i in range(heads * vd)], f32)
    s0 = np.array([(i - 7.0) / 31.0 for i in range(heads * kd * vd)], f32)
    g, beta = np.array([-0.2, -0.4], f32), np.array([0.3, 0.7], f32)
    exp_out, exp_state = _strided_reference(q, k, v, g, beta, heads, kd, vd, s0)
    out, state = oracle.delta_step(q, k, v, g, beta, heads, kd, vd, s0)
    assert np.abs(out - exp_out).max() < 1e-6
    assert np.abs(state - exp_state).max() < 1e-6


def test_flat_causal_convolution_matches_row_reference():
    """src/qwen/quantized_deltanet.rs:869-896: three channels, kernel 3;
    output and rolled state bit-identical to the row-by-row reference."""
    inp = np.array([0.25, -0.5, 1.25], f32)
    w = np.array([0.1, 0.2, -0.3, 0.4, -0.2, 0.3, 0.5, -0.7, 0.6], f32)
    state = np.array([0.75, -0.25, 0.5, 1.0, -1.5, 0.2], f32)
    exp_state, exp_out = state.copy(), np.zeros(3, f32)
    for ch in range(3):
        hist, row = exp_state[ch * 2:ch * 2 + 2], w[ch * 3:ch * 3 + 3]
        s = f32(row[2] * inp[ch])
        for tap in range(2):
            s = f32(s + f32(row[tap] * hist[tap]))
        sig = f32(f32(1) / f32(f32(1) + np.exp(-s, dtype=f32)))
        exp_out[ch] = f32(s * sig)
    for ch in range(3):
        hist = exp_state[ch * 2:ch * 2 + 2]
        hist[0], hist[1] = hist[1], inp[ch]
    out, new_state = oracle.conv_step(inp, w, 3, state)
    assert np.array_equal(out, exp_out)
    assert np.array_equal(new_state, exp_state)


def test_gguf_state_scale_is_already_negative_exp_a_log():
    """quantized_deltanet.rs:898-906: ssm_a holds -exp(A_log)."""
    a_log, alpha, bias = f32(1.5), f32(0.25), f32(-0.1)
    gguf_value = -np.exp(a_log, dtype=f32)
    sp = oracle.softplus(float(f32(alpha + bias)))
    reference = -np.exp(a_log, dtype=f32) * f32(np.log1p(np.exp(np.float64(f32(alpha + bias)))))
    assert abs(gguf_value * f32(sp) - reference) < 1e-6


def test_value_head_layout_matches_grouped_and_tiled_gguf_orders():
    """quantized_deltanet.rs:908-920: two key heads, two repeats."""
    grouped = [oracle.value_head(k, r, 2, 2, False) for k in range(2) for r in range(2)]
    tiled = [oracle.value_head(k, r, 2, 2, True) for k in range(2) for r in range(2)]
    assert grouped == [0, 1, 2, 3]
    assert tiled == [0, 2, 1, 3]


def test_router_selects_and_normalizes_top_k():
    """src/qwen/moe.rs:232-238: logits [1, 4, 2, 3], top-2 -> experts
    [1, 3], weights summing to one."""
    experts, weights = oracle.route([1, 4, 2, 3], 2, True)
    assert list(experts) == [1, 3]
    assert abs(float(weights.sum()) - 1) < 1e-6


def test_converted_gguf_norm_matches_one_centered_hf_norm():
    """src/qwen/quantized_layer.rs:245-259 and src/qwen/norm.rs:7-14: the GGUF
    norm with weight 1 + w equals the HF norm with weight w, exactly."""
    x = np.array([2, -3, 4], f32)
    hf_w = np.array([0.1, -0.2, 0.3], f32)
    var = f32(f32(x[0] * x[0]) + f32(x[1] * x[1]))
    var = f32(var + f32(x[2] * x[2])) * f32(1.0 / 3.0)
    den = np.sqrt(f32(var + f32(1e-6)), dtype=f32)
    hf = (x / den).astype(f32) * (hf_w + f32(1)).astype(f32)
    assert np.array_equal(oracle.rms_norm(x, hf_w + f32(1), 1e-6), hf.astype(f32))


def test_converted_qk_norm_uses_weight_without_second_offset():
    """src/qwen/quantized_attention.rs:857-864: [3, 4] with weight [2, 3],
    eps 0 -> [6, 12] / sqrt(12.5)."""
    out = oracle.converted_norm([3, 4], [2, 3], 0.0)
    rms = np.sqrt(f32(12.5))
    assert abs(out[0] - 6 / rms) < 1e-6 and abs(out[1] - 12 / rms) < 1e-6


def test_the_dot_sums_its_lanes_in_a_fixed_order():
    """quantized_attention.rs:883-906: with exact arithmetic the lane dot
    equals the serial sum; a ragged width consumes every element; the same
    inputs give the same bits."""
    q = np.arange(256, dtype=f32)
    k = (np.arange(256) % 7).astype(f32)
    assert oracle.dot8(q, k) == float(np.sum(q * k, dtype=np.float64))
    assert oracle.dot8(np.ones(11, f32), np.arange(11, dtype=f32)) == 55.0
    assert oracle.dot8([], []) == 0.0
    for n in (8, 64, 256, 300):
        a, b = np.sin(np.arange(n)).astype(f32), np.cos(np.arange(n)).astype(f32)
        assert oracle.dot8(a, b) == oracle.dot8(a, b)


def _wave(seed, index):
    """scan_fixture's cheap deterministic values (quantized_attention.rs:941-977)."""
    bits = int(np.array(seed, f32).view(np.uint32))
    rot = ((bits << 11) | (bits >> 21)) & 0xFFFFFFFF
    mixed = (np.asarray(index, np.uint64) * 2654435761 + rot) & 0xFFFFFFFF
    return ((mixed >> 9) % 4096).astype(f32) / f32(2048) - f32(1)


@pytest.mark.parametrize("existing,nh,nkv,hd", [(5, 8, 2, 24), (613, 8, 2, 24), (4096, 16, 2, 256)])
def test_scan_matches_a_float64_scan_at_the_reference_geometries(existing, nh, nkv, hd):
    """The geometries of quantized_attention.rs:979-1036 (blocked == per-head
    scan, including 16 query / 2 KV heads at head_dim 256 against 4096 cached
    positions) on the reference's own fixture values: the oracle's per-head
    scan (dot8 scores, softmax with a divide, sigmoid gate, head h reading KV
    head h / (nh / nkv)) within 1e-5 of the same scan in float64."""
    cached = existing + 1
    q = np.stack([_wave(f32(0.37) + f32(h * 0.11), np.arange(hd)) for h in range(nh)])
    gate = np.stack([_wave(f32(0.91) + f32(h * 0.11), np.arange(hd)) for h in range(nh)])
    keys = _wave(f32(0.013), np.arange(cached * nkv * hd)).reshape(cached, nkv, hd)
    values = _wave(f32(0.029), np.arange(cached * nkv * hd)).reshape(cached, nkv, hd)
    out = oracle.attend(q, gate, keys, values, nh, nkv, hd).reshape(nh, hd)
    g = nh // nkv
    for h in range(nh):
        kk, vv = keys[:, h // g].astype(np.float64), values[:, h // g].astype(np.float64)
        sc = kk @ q[h].astype(np.float64) / np.sqrt(hd)
        p = np.exp(sc - sc.max())
        p /= p.sum()
        ref = (p @ vv) / (1 + np.exp(-gate[h].astype(np.float64)))
        assert np.abs(out[h] - ref).max() < 1e-5, h


def test_verifier_accepts_only_the_matching_draft_prefix():
    """src/runtime.rs:2392-2398."""
    logits = np.array([[0, 3, 1], [4, 0, 1], [0, 1, 5]], f32)
    assert oracle.accepted_prefix([1, 2], logits) == 1
    assert oracle.accepted_prefix([1], logits[:2]) == 1
    assert oracle.accepted_prefix([], logits[:1]) == 0


def test_mtp_hidden_inputs_shift_target_rows_by_one_position():
    """src/runtime.rs:2382-2390, through libiq's host-side builder of the
    MTP catch-up inputs (iq_mtp_shifted_inputs)."""
    L = _lib.lib()
    L.iq_mtp_shifted_inputs.argtypes = [ctypes.c_void_p] * 2 + [ctypes.c_int] * 2 + [ctypes.c_void_p]
    hidden = np.array([[1, 2], [3, 4], [5, 6]], f32)
    prev = np.array([9, 8], f32)
    out = np.empty((3, 2), f32)
    assert L.iq_mtp_shifted_inputs(prev.ctypes.data, hidden.ctypes.data, 3, 2, out.ctypes.data) == 0
    assert out.tolist() == [[9, 8], [1, 2], [3, 4]]
    assert L.iq_mtp_shifted_inputs(None, hidden.ctypes.data, 2, 2, out.ctypes.data) == 0
    assert out[:2].tolist() == [[0, 0], [1, 2]]
