"""Greedy decoding with speculative verification (the reference's speculative decode: its verify section,
agxforge/inference/assemble.py:244-253,747-803, driven by tools/g17specgen.m with prompt-lookup drafts).

    prompt_lookup(history, ngram=3, min_ngram=2, max_draft=15)
        the draft: the longest suffix of `history` (ngram down to min_ngram tokens) that occurred earlier in it,
        and the tokens that followed its most recent earlier occurrence (at most max_draft)
    generate(model, tokens, b=0, ngram=3, min_ngram=2, max_draft=15)
        `tokens` greedy tokens of sequence b: every round drafts from the sequence's own history (its token log) and
        verifies the draft in one pass of rows (DecodeModel.verify: the accepted drafts plus the model's next choice);
        with no draft, one ordinary decode step. Returns (tokens, rounds, drafted, accepted).

Greedy verification emits the tokens greedy decoding chooses (the rows' choices are the first maxima of their own
logits), computed in fewer passes when drafts are accepted; the row pass sums in the tensor-core GEMMs' order, so the
logits agree with the decode step's within rounding.
"""
from __future__ import annotations

import numpy as np


def prompt_lookup(history, ngram=3, min_ngram=2, max_draft=15):
    h = [int(t) for t in history]
    for n in range(min(ngram, len(h) - 1), min_ngram - 1, -1):
        if n <= 0:
            break
        key = h[-n:]
        for start in range(len(h) - n - 1, -1, -1):   # the most recent earlier occurrence
            if h[start:start + n] == key:
                follow = h[start + n:start + n + max_draft]
                if follow:
                    return follow
    return []


def generate(model, tokens, b=0, ngram=3, min_ngram=2, max_draft=15):
    out = []
    rounds = drafted = accepted = 0
    while len(out) < tokens:
        q0, log = model.state(b)
        hist = [int(t) for t in log[: q0 + 1]]
        room = min(max_draft, tokens - len(out) - 1, model.cap - q0 - 2)
        draft = prompt_lookup(hist, ngram, min_ngram, room) if room > 0 else []
        rounds += 1
        if draft:
            emitted, _ = model.verify(draft, b)
            drafted += len(draft)
            accepted += len(emitted) - 1
        else:
            toks, _, _ = model.decode(1, want_tokens=True)
            emitted = [int(toks[0, b])]
        out.extend(emitted)
    return out[:tokens], rounds, drafted, accepted
