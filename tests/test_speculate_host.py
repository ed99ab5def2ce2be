"""The prompt-lookup draft on the CPU (agxforge.inference.speculate.prompt_lookup): the longest repeated suffix's
most recent continuation, bounded by max_draft, none when nothing repeats."""
from agxforge.inference.speculate import prompt_lookup


def test_prompt_lookup():
    h = [1, 2, 3, 4, 5, 9, 2, 3, 4]
    assert prompt_lookup(h, ngram=3, min_ngram=2, max_draft=15) == [5, 9, 2, 3, 4]
    assert prompt_lookup(h, max_draft=2) == [5, 9]
    assert prompt_lookup([1, 2, 3, 4], ngram=3, min_ngram=2) == []
    # the most recent earlier occurrence wins
    assert prompt_lookup([7, 8, 1, 7, 8, 2, 7, 8], ngram=2, min_ngram=2) == [2, 7, 8]
    assert prompt_lookup([5], ngram=3) == []
