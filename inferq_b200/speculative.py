"""Host side of speculative decoding over libiq: the policy loop the
reference runtime drives around the device pass.

``MtpLoop`` restates the MTP generation loop of src/runtime.rs:1563-1952:
``draft_mtp`` (:1995-2056; depth drafts from the MTP head against the
vocabulary-prefix LM head, stopping before the first below ``min_conf``),
``verify_rows`` + ``accepted_draft_prefix`` + rollback (:2102-2114,
:2225-2236; one iq_verify), then ``synchronize_mtp`` (:2058-2088) over the
committed rows.  ``NgramIndex`` restates the prompt-lookup index of
src/ngram.rs (the most recent verified occurrence of the longest suffix key
proposes its continuation) and ``NgramLoop`` drives it at a fixed draft
width.  The reference's adaptive draft-length controller
(src/speculative.rs) is host policy that the Rust runtime keeps.
"""
from __future__ import annotations

import numpy as np

from .model import State


class MtpLoop:
    """Greedy speculative decoding with the MTP draft head."""

    def __init__(self, state: State, depth: int = 3, draft_vocab: int = 32768, min_conf: float = 0.0):
        self.state = state
        self.depth = depth
        self.draft_vocab = min(draft_vocab, state.model.cfg.vocab_size)
        self.min_conf = min_conf
        self.seed = None          # next token to evaluate (already emitted)
        self.prev_hidden = None   # target hidden row of the position before `seed`
        self.position = 0         # target position of `seed`
        self.last = {}

    def prefill(self, prompt) -> int:
        """Evaluate the prompt, build the MTP cache over it; returns the first
        generated token."""
        am, _, hidden = self.state.forward(prompt, hidden=True)
        self.state.mtp_sync(0, None, prompt, hidden)
        self.seed = int(am[-1])
        self.prev_hidden = np.ascontiguousarray(hidden[-1])
        self.position = len(prompt)
        return self.seed

    def step(self) -> list[int]:
        """One draft -> verify -> catch-up round; returns the newly emitted
        tokens (accepted drafts, then the authoritative token)."""
        st = self.state
        toks, probs, margins, n = st.mtp_draft(self.seed, self.prev_hidden, self.depth, self.draft_vocab,
                                               self.min_conf)
        drafts = [int(t) for t in toks[:n]]
        (acc, auth, com), _, hid = st.verify([self.seed] + drafts, hidden=True)
        committed = [self.seed] + drafts[:acc]
        st.mtp_sync(self.position, self.prev_hidden, committed, hid[:com])
        self.position += com
        self.prev_hidden = np.ascontiguousarray(hid[acc])
        self.seed = int(auth)
        H = st.model.cfg.hidden_size
        rows = 1 + len(drafts)
        self.last = {"drafted": len(drafts), "accepted": acc, "committed": com,
                     # bytes crossing PCIe in this round (tokens, hidden rows, results)
                     "h2d": 4 + 4 * H + 4 * rows + 4 * com + 4 * com * H,
                     "d2h": 3 * 16 * 4 + 16 + 4 * rows * H}
        return drafts[:acc] + [int(auth)]


INDEXED_MATCH_LENGTHS = (4, 3, 2)
MAX_MATCH_LEN, MIN_MATCH_LEN = 4, 2


def fnv1a_tokens(tokens) -> int:
    """FNV-1a over the raw token ids (src/ngram.rs:29-36)."""
    h = 0xCBF29CE484222325
    for t in tokens:
        h ^= int(t)
        h = (h * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


class NgramIndex:
    """Incremental n-gram index over the tokens in context (NgramIndex,
    src/ngram.rs:58-234): one map per key length 4, 3, 2 holding the most
    recent end position of each key; ``push`` records, per length, the
    occurrence the map held before this token (the most recent earlier
    occurrence of the new suffix); a lookup compares the actual tokens, so a
    hash collision is a miss, never a wrong draft."""

    def __init__(self, hasher=fnv1a_tokens):
        self.hasher = hasher
        self.clear()

    def clear(self):
        self.tokens = []
        self.maps = [dict() for _ in INDEXED_MATCH_LENGTHS]
        self.last_match = [None] * len(INDEXED_MATCH_LENGTHS)

    def __len__(self):
        return len(self.tokens)

    def extend(self, tokens):
        for t in tokens:
            self.push(t)

    def push(self, token: int):
        self.tokens.append(int(token))
        end = len(self.tokens) - 1
        for slot, n in enumerate(INDEXED_MATCH_LENGTHS):
            if len(self.tokens) < n:
                self.last_match[slot] = None
                continue
            key = self.hasher(self.tokens[-n:])
            self.last_match[slot] = self.maps[slot].get(key)
            self.maps[slot][key] = end

    def most_recent_match(self, match_len: int):
        if match_len not in INDEXED_MATCH_LENGTHS:
            return None
        cand = self.last_match[INDEXED_MATCH_LENGTHS.index(match_len)]
        if cand is None or cand + 1 < match_len or cand >= len(self.tokens):
            return None
        earlier = self.tokens[cand + 1 - match_len:cand + 1]
        return cand if earlier == self.tokens[-match_len:] else None

    def draft(self, draft_len: int, min_match: int, is_stop=lambda t: False):
        """Up to ``draft_len`` continuation tokens of the longest verified key
        (lengths tried longest first down to ``min_match``), truncated at the
        first stop token; None on a miss.  Returns (tokens, match_len,
        source_position, truncated_at_stop)."""
        if draft_len == 0:
            return None
        min_match = max(MIN_MATCH_LEN, min(MAX_MATCH_LEN, min_match))
        for n in INDEXED_MATCH_LENGTHS:
            if n < min_match:
                continue
            pos = self.most_recent_match(n)
            if pos is None:
                continue
            start, end = pos + 1, min(pos + 1 + draft_len, len(self.tokens))
            if start >= end:
                continue
            cand = self.tokens[start:end]
            stop = next((i for i, t in enumerate(cand) if is_stop(t)), None)
            toks = cand[:stop] if stop is not None else cand
            if not toks:
                return None
            return toks, n, pos, stop is not None
        return None


class NgramLoop:
    """Greedy n-gram speculative decoding (the ngram policy of
    src/speculative.rs over src/ngram.rs): draft up to k-1 tokens from the
    index, verify [seed, drafts] in one pass, commit the accepted prefix and
    the authoritative token."""

    def __init__(self, state: State, k: int = 4, min_match: int = 4):
        # min_match 4: DEFAULT_NGRAM_MIN_MATCH (src/runtime.rs:297)
        self.state, self.k, self.min_match = state, k, min_match
        self.index = NgramIndex()
        self.seed = None
        self.last = {}

    def prefill(self, prompt) -> int:
        am, _, _ = self.state.forward(prompt)
        self.index.extend(prompt)
        self.seed = int(am[-1])
        return self.seed

    def step(self) -> list[int]:
        self.index.push(self.seed)
        d = self.index.draft(self.k - 1, self.min_match)
        drafts = list(d[0]) if d else []
        (acc, auth, com), _, _ = self.state.verify([self.seed] + drafts)
        self.index.extend(drafts[:acc])
        self.seed = int(auth)
        self.last = {"drafted": len(drafts), "accepted": acc, "committed": com,
                     "h2d": 4 * (1 + len(drafts)), "d2h": 16}
        return drafts[:acc] + [int(auth)]
