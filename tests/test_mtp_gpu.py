"""The MTP draft head on the device against the CPU oracle and against itself.

The oracle restates QuantizedMtpHead::forward_with_head
(src/qwen/quantized_mtp.rs:175-227) one row at a time; catch-up follows
synchronize_mtp / shifted_hidden_inputs (src/runtime.rs:2058-2088,
:2184-2223) and drafting draft_mtp + top1_with_scores (:1995-2056,
:2245-2265).
"""
import numpy as np
import pytest

import oracle
from inferq_b200 import synth
from inferq_b200.model import Model, State

pytestmark = pytest.mark.gpu

TOL = 2e-2


@pytest.fixture(scope="module")
def pair(cuda):
    cfg = synth.mini_35b()
    assert cfg.mtp_num_hidden_layers == 1
    tensors = list(synth.generate(cfg, seed=5))
    return cfg, Model(cfg, tensors), oracle.OracleModel(cfg, tensors)


def _oracle_draft(om, cfg, prompt, hidden, seed, depth, vocab):
    """Oracle: target hidden rows given, catch-up over the prompt, then drafting."""
    st = om.state(256)
    H = cfg.hidden_size
    for i, t in enumerate(prompt):
        st.mtp(int(t), hidden[i - 1] if i else np.zeros(H, np.float32), 0)
    tok, h = seed, hidden[len(prompt) - 1]
    out = []
    for _ in range(depth):
        lg, h = st.mtp(tok, h, vocab)
        top = oracle.argmax(lg)
        peak = lg[top]
        second = np.max(np.delete(lg, top))
        prob = 1.0 / np.sum(np.exp((lg - peak).astype(np.float64)))
        out.append((top, float(peak - second), float(prob)))
        tok = top
    return out


def test_mtp_drafts_match_the_oracle(pair):
    cfg, model, om = pair
    prompt = np.random.default_rng(2).integers(0, cfg.vocab_size, 12)
    st = State(model, 256)
    am, _, hid = st.forward(prompt, hidden=True)
    st.mtp_sync(0, None, prompt, hid)
    assert st.mtp_position == len(prompt)
    vocab = cfg.vocab_size // 2  # a vocabulary-prefix head
    seed = int(am[-1])
    tok, prob, margin, n = st.mtp_draft(seed, hid[-1], 3, vocab)
    ref = _oracle_draft(om, cfg, prompt, hid, seed, 3, vocab)
    assert st.mtp_position == len(prompt) + 3
    for i, (rt, rm, rp) in enumerate(ref):
        if i and int(tok[i - 1]) != ref[i - 1][0]:
            break  # the chains diverged on a near tie; later steps differ
        # top-1 probability within 2% (relative), logit margin within TOL
        assert abs(prob[i] - rp) <= 2e-2 * rp, (i, prob, ref)
        assert abs(margin[i] - rm) <= TOL, (i, margin, ref)
        if rm > 4 * TOL:
            assert int(tok[i]) == rt, (i, tok, ref)
    assert n == 3  # min_conf 0 keeps every draft


def test_draft_threshold_counts_the_confident_prefix(pair):
    cfg, model, _ = pair
    prompt = np.random.default_rng(3).integers(0, cfg.vocab_size, 6)
    st = State(model, 256)
    am, _, hid = st.forward(prompt, hidden=True)
    st.mtp_sync(0, None, prompt, hid)
    tok, prob, _, n = st.mtp_draft(int(am[-1]), hid[-1], 4, cfg.vocab_size, min_conf=2.0)
    assert n == 0  # no probability reaches 2
    st.mtp_sync(len(prompt), hid[-1], [int(am[-1])], hid[-1:])
    tok2, prob2, _, n2 = st.mtp_draft(int(tok[0]), hid[-1], 4, cfg.vocab_size, min_conf=0.0)
    assert n2 == 4
    thr = float(prob2[1])
    st.mtp_sync(len(prompt), hid[-1], [int(am[-1])], hid[-1:])
    # same position and inputs as the previous call: the same drafts, and
    # min_conf between step 1's and step 0's probability cuts after step 0
    tok3, prob3, _, n3 = st.mtp_draft(int(tok[0]), hid[-1], 4, cfg.vocab_size, min_conf=thr + 1e-6)
    assert np.array_equal(tok3, tok2) and np.array_equal(prob3, prob2)
    expect = 0
    while expect < 4 and prob3[expect] >= thr + 1e-6:
        expect += 1
    assert n3 == expect


def test_catch_up_in_pieces_equals_one_catch_up(pair):
    """Multi-row MTP rows are bitwise the rows of sequential catch-ups."""
    cfg, model, _ = pair
    prompt = np.random.default_rng(4).integers(0, cfg.vocab_size, 11)
    ref = State(model, 256)
    am, _, hid = ref.forward(prompt, hidden=True)
    a, b = State(model, 256), State(model, 256)
    a.forward(prompt)
    b.forward(prompt)
    a.mtp_sync(0, None, prompt, hid)
    b.mtp_sync(0, None, prompt[:4], hid[:4])
    b.mtp_sync(4, hid[3], prompt[4:9], hid[4:9])
    b.mtp_sync(9, hid[8], prompt[9:], hid[9:])
    da = a.mtp_draft(int(am[-1]), hid[-1], 3, cfg.vocab_size)
    db = b.mtp_draft(int(am[-1]), hid[-1], 3, cfg.vocab_size)
    for x, y in zip(da[:3], db[:3]):
        assert np.array_equal(np.asarray(x).view(np.uint32), np.asarray(y).view(np.uint32))


def test_sync_truncates_speculative_mtp_rows(pair):
    """Drafting appends speculative MTP rows; the next catch-up drops them."""
    cfg, model, _ = pair
    prompt = np.random.default_rng(6).integers(0, cfg.vocab_size, 7)
    st = State(model, 256)
    am, _, hid = st.forward(prompt, hidden=True)
    st.mtp_sync(0, None, prompt, hid)
    first = st.mtp_draft(int(am[-1]), hid[-1], 3, cfg.vocab_size)
    assert st.mtp_position == len(prompt) + 3
    st.mtp_sync(len(prompt), hid[-1], [int(am[-1])], hid[-1:])
    assert st.mtp_position == len(prompt) + 1
    fresh = State(model, 256)
    fresh.forward(prompt)
    fresh.mtp_sync(0, None, list(prompt) + [int(am[-1])], np.concatenate([hid, hid[-1:]]))
    x = st.mtp_draft(int(first[0][0]), hid[-1], 2, cfg.vocab_size)
    y = fresh.mtp_draft(int(first[0][0]), hid[-1], 2, cfg.vocab_size)
    assert np.array_equal(x[0], y[0]) and np.array_equal(x[1].view(np.uint32), y[1].view(np.uint32))
