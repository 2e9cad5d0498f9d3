"""NGramIndex semantics, restating the reference's model-free lookup tests
(tests/test_lookup.py:14-66) on the same token sequences."""
from mlx_dspark_b200.lookup import NGramIndex


def _idx(tokens, **kw):
    ix = NGramIndex(**kw)
    ix.extend(list(tokens))
    return ix


def test_default_minimum_is_trigram():
    assert _idx([5, 6, 7, 0, 1, 2, 5, 6]).propose() == []
    assert _idx([4, 5, 6, 7, 8, 0, 4, 5, 6], max_draft=2).propose() == [7, 8]


def test_no_match_returns_empty():
    assert _idx([1, 2, 3, 4]).propose() == []


def test_simple_repeat_proposes_continuation():
    assert _idx([5, 6, 7, 8, 9, 1, 5, 6], min_n=2, max_n=3, max_draft=3).propose() == [7, 8, 9]


def test_self_occurrence_is_skipped():
    assert _idx([1, 2, 3, 4, 5], min_n=2, max_n=3).propose() == []


def test_latest_earlier_occurrence_wins():
    assert _idx([5, 6, 7, 0, 5, 6, 8, 0, 5, 6], min_n=2, max_n=3, max_draft=1).propose() == [8]


def test_longer_ngram_preferred():
    assert _idx([4, 5, 6, 9, 0, 5, 6, 7, 0, 4, 5, 6], min_n=2, max_n=3, max_draft=1).propose() == [9]


def test_max_draft_and_tail_truncation():
    assert _idx([5, 6, 7, 8, 9, 10, 11, 0, 5, 6], min_n=2, max_n=3, max_draft=4).propose() == [7, 8, 9, 10]
    assert _idx([1, 9, 9, 2, 9, 9], min_n=2, max_n=3, max_draft=4).propose() == [2, 9, 9]


def test_incremental_extend_matches_bulk():
    toks = [3, 1, 4, 1, 5, 9, 2, 6, 5, 3, 5, 9]
    bulk = _idx(toks, min_n=2, max_n=3, max_draft=2)
    inc = NGramIndex(min_n=2, max_n=3, max_draft=2)
    for t in toks:
        inc.extend([t])
    assert bulk.propose() == inc.propose()
