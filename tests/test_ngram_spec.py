"""N-gram lookup drafts (host logic)."""


def test_ngram_draft_longest_recent_match():
    from swarmllm_b200.engine.ngram_spec import ngram_draft
    ctx = [1, 2, 3, 4, 5, 9, 2, 3, 7, 8, 1, 2, 3]
    # suffix (1, 2, 3) occurred at 0: what followed was 4, 5, 9
    assert ngram_draft(ctx, 3, 3) == [4, 5, 9]
    # suffix 2-gram (2, 3) most recently at 6 -> 7, 8 ... when 3-grams are off
    assert ngram_draft(ctx, 2, 2) == [7, 8]
    assert ngram_draft([5, 6, 7], 3, 4) == []               # nothing repeats
    assert ngram_draft([4, 4], 3, 3) == [4]                  # a 1-gram match
    assert ngram_draft([1], 3, 3) == []
    assert ngram_draft(ctx, 3, 0) == []
