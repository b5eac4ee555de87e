"""The speculative loops' host bookkeeping (inferq_b200/speculative.py) on
CPU, over a fake state whose "model" is a fixed next-token rule.

The fake keeps the device contract of iq_verify: the rows are
[seed, drafts...], the accepted count is the longest draft prefix equal to
the target's own greedy tokens (accepted_draft_prefix, src/runtime.rs:2382-
2398), the authoritative token is the target's token after the last
accepted row, and only the committed rows stay in the state.  Against it:

* both loops emit exactly the plain greedy sequence, whatever the drafts;
* MtpLoop's catch-up covers every committed position once, in order, with
  the MTP block's shifted inputs (token p with the target hidden row of
  position p-1, src/runtime.rs:2058-2088 synchronize_mtp);
* the per-round counts (drafted, accepted, committed) agree with the tokens
  returned.
"""
import numpy as np
import pytest

from inferq_b200.speculative import MtpLoop, NgramLoop

V, H = 97, 4


def greedy_next(t):
    return (7 * int(t) + 3) % V


class _Cfg:
    vocab_size = V
    hidden_size = H


class _Model:
    cfg = _Cfg()


class FakeState:
    """Committed tokens and positions; hidden row of position p = [p, tok, 0, 0]."""

    def __init__(self, seed=0, corrupt=0.3, short=0.0):
        self.model = _Model()
        self.tokens = []
        self.synced = []          # (position, prev_hidden, tokens, target_hidden) per mtp_sync call
        self.rng = np.random.default_rng(seed)
        self.corrupt, self.short = corrupt, short

    def _hidden(self, start, toks):
        return np.array([[start + i, t, 0.0, 0.0] for i, t in enumerate(toks)], np.float32).reshape(-1, H)

    def forward(self, tokens, *, logits=False, hidden=False):
        start = len(self.tokens)
        self.tokens += [int(t) for t in tokens]
        am = np.array([greedy_next(t) for t in tokens], np.int32)
        return am, None, self._hidden(start, tokens) if hidden else None

    def verify(self, tokens, *, logits=False, hidden=False):
        start = len(self.tokens)
        rows = [int(t) for t in tokens]
        acc = 0
        while acc + 1 < len(rows) and rows[acc + 1] == greedy_next(rows[acc]):
            acc += 1
        self.tokens += rows[:acc + 1]  # the rejected rows are rolled back
        hd = self._hidden(start, rows) if hidden else None
        return (acc, greedy_next(rows[acc]), acc + 1), None, hd

    def mtp_sync(self, position, prev_hidden, tokens, target_hidden):
        self.synced.append((position, None if prev_hidden is None else np.array(prev_hidden),
                            [int(t) for t in tokens], np.array(target_hidden)))

    def mtp_draft(self, seed, hidden, depth, draft_vocab, min_conf=0.0):
        toks, t = [], seed
        for _ in range(depth):
            t = greedy_next(t)
            if self.rng.random() < self.corrupt:
                t = int(self.rng.integers(draft_vocab))
            toks.append(t)
        n = depth if self.rng.random() >= self.short else int(self.rng.integers(depth + 1))
        return np.array(toks, np.int32), np.ones(depth, np.float32), np.ones(depth, np.float32), n


def _greedy(prompt, n):
    out = [greedy_next(prompt[-1])]
    while len(out) < n:
        out.append(greedy_next(out[-1]))
    return out


@pytest.mark.parametrize("corrupt,short", [(0.0, 0.0), (0.3, 0.0), (0.6, 0.3), (1.0, 0.0)])
def test_mtp_loop_emits_plain_greedy_and_syncs_every_position(corrupt, short):
    st = FakeState(seed=int(corrupt * 10), corrupt=corrupt, short=short)
    loop = MtpLoop(st, depth=3, draft_vocab=64)
    prompt = [5, 9, 13, 2, 40]
    emitted = [loop.prefill(prompt)]
    accepted = []
    for _ in range(40):
        toks = loop.step()
        last = loop.last
        assert len(toks) == last["committed"] == last["accepted"] + 1
        assert last["accepted"] <= last["drafted"] <= 3
        accepted.append(last["accepted"])
        emitted += toks
    assert emitted == _greedy(prompt, len(emitted))
    if corrupt == 0.0 and short == 0.0:
        assert all(a == 3 for a in accepted)
    if corrupt == 1.0:
        assert sum(accepted) <= 2  # a random draft equal to greedy by chance only
    # the state holds prompt + every committed token, nothing rejected
    assert st.tokens == prompt + emitted[:-1]
    # catch-up: contiguous positions, each token with the previous position's hidden row
    pos = 0
    for position, prev, toks, hid in st.synced:
        assert position == pos
        if position == 0:
            assert prev is None
        else:
            assert prev[0] == position - 1 and prev[1] == st.tokens[position - 1]
        assert toks == st.tokens[position:position + len(toks)]
        assert np.array_equal(hid[:, 0], np.arange(position, position + len(toks)))
        assert np.array_equal(hid[:, 1], np.array(toks, np.float32))
        pos += len(toks)
    assert pos == len(st.tokens)


def test_ngram_loop_emits_plain_greedy_on_a_repeating_prompt():
    # a prompt made of the greedy rule's own cycle, twice: once past the
    # first lap the index proposes exactly the greedy continuation
    cyc = [1]
    while greedy_next(cyc[-1]) != cyc[0]:
        cyc.append(greedy_next(cyc[-1]))
    prompt = cyc * 2
    st = FakeState()
    loop = NgramLoop(st, k=8)
    emitted = [loop.prefill(prompt)]
    accepted = []
    for _ in range(20):
        toks = loop.step()
        assert len(toks) == loop.last["committed"] == loop.last["accepted"] + 1
        assert loop.last["drafted"] <= 7
        accepted.append(loop.last["accepted"])
        emitted += toks
    assert emitted == _greedy(prompt, len(emitted))
    assert st.tokens == prompt + emitted[:-1]
    assert accepted == [7] * 20  # every draft of the cycle is the greedy continuation


def test_ngram_loop_without_matches_commits_one_token_per_step():
    prompt = list(range(10, 30))  # no repetition: nothing to draft
    st = FakeState()
    loop = NgramLoop(st, k=8)
    emitted = [loop.prefill(prompt)]
    toks = loop.step()
    assert loop.last["drafted"] == 0 and toks == [greedy_next(emitted[0])]
