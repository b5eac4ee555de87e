"""The n-gram drafter's index, against the reference's own tests
(src/ngram.rs:243-349), on the CPU."""
from inferq_b200.speculative import NgramIndex


def index_of(tokens, hasher=None):
    ix = NgramIndex(hasher) if hasher else NgramIndex()
    ix.extend(tokens)
    return ix


def test_lookup_returns_the_most_recent_prior_occurrence():
    ix = index_of([1, 2, 3, 9, 1, 2, 3, 8, 1, 2, 3])
    assert ix.most_recent_match(3) == 6 and ix.most_recent_match(2) == 6


def test_draft_continues_from_the_most_recent_occurrence():
    ix = index_of([1, 2, 3, 40, 41, 42, 9, 1, 2, 3, 50, 51, 52, 1, 2, 3])
    toks, _, pos, _ = ix.draft(3, 3)
    assert toks == [50, 51, 52] and ix.tokens[pos] == 3


def test_longer_keys_are_preferred_over_shorter_ones():
    ix = index_of([7, 2, 3, 60, 5, 2, 3, 70, 7, 2, 3])
    toks, n, _, _ = ix.draft(1, 3)
    assert n == 3 and toks == [60]
    assert ix.draft(1, 2)[1] == 3


def test_min_match_two_finds_matches_a_trigram_key_would_miss():
    ix = index_of([4, 5, 99, 1, 2, 4, 5])
    assert ix.draft(2, 3) is None
    toks, n, _, _ = ix.draft(2, 2)
    assert n == 2 and toks == [99, 1]


def test_draft_truncates_at_the_first_stop_token():
    toks, _, _, trunc = index_of([1, 2, 3, 40, 41, 77, 42, 1, 2, 3]).draft(5, 3, lambda t: t == 77)
    assert toks == [40, 41] and trunc


def test_draft_is_empty_when_the_continuation_starts_with_a_stop_token():
    assert index_of([1, 2, 3, 77, 40, 1, 2, 3]).draft(5, 3, lambda t: t == 77) is None


def test_a_sequence_without_repetition_drafts_nothing():
    ix = index_of([1, 2, 3, 4, 5, 6, 7, 8])
    assert ix.draft(4, 3) is None and ix.draft(4, 2) is None


def test_hash_collisions_are_rejected_by_comparing_token_ids():
    zero = lambda toks: 0
    ix = index_of([1, 2, 3, 40, 41, 42, 7, 8, 9], zero)
    assert ix.most_recent_match(3) is None and ix.draft(4, 3) is None
    ow = index_of([1, 2, 3, 40, 41, 1, 2, 3], zero)
    assert ow.most_recent_match(3) is None and ow.draft(2, 3) is None
    per = index_of([5, 5, 5, 5], zero)
    assert per.most_recent_match(3) == 2 and per.draft(1, 3)[0] == [5]


def test_draft_is_clamped_to_the_tokens_that_exist():
    assert index_of([1, 2, 3, 40, 1, 2, 3]).draft(8, 3)[0] == [40, 1, 2, 3]


def test_clear_drops_every_indexed_position():
    ix = index_of([1, 2, 3, 40, 1, 2, 3])
    ix.clear()
    assert len(ix) == 0 and ix.most_recent_match(3) is None
    ix.extend([1, 2, 3])
    assert ix.most_recent_match(3) is None


def test_zero_draft_length_proposes_nothing():
    assert index_of([1, 2, 3, 40, 1, 2, 3]).draft(0, 3) is None
