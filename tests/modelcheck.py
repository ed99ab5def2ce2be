"""Shared helpers of the model-level parity tests (test infrastructure): build a device model with its packs kept,
mirror it into the CPU oracle, run a teacher-forced decode on the GPU and compare every step's logits with the FP64
oracle (the reference's bound 0.05 + 0.003*|ref|, tools/g17generationcheck.py:39) and its argmax with the
half-transport oracle's."""
from __future__ import annotations

import numpy as np

from oracle import decoder as D


def oracle_model(m):
    """The CPU oracle's copy of a DecodeModel built with keep_packs=True."""
    S = m.shape
    shape = D.Shape(S.D_MODEL, S.LAYERS, S.HEADS, S.KV_HEADS, S.HEAD_DIM, S.FFN, S.VOCAB, S.EPS, S.ROPE_THETA,
                    S.QKV_BIAS, S.TIED)
    k = m.packs
    bits, sdt = m.bits, m.cfg["scale_dtype"]

    def pack(key, n, kk):
        a, s, b = k[key]
        return D.Pack(a, s, b, bits, sdt, n, kk)

    layers = []
    for l in range(S.LAYERS):
        L = {}
        for role, n, kk in S.matrices():
            L[role] = pack((l, role), n, kk)
        L["g1"] = k[(l, "attn_gain")]
        L["g2"] = k[(l, "ffn_gain")]
        L["bias"] = k.get((l, "qkv_bias"))
        layers.append(L)
    head = pack((None, "head"), S.VOCAB, S.D_MODEL)
    return D.Model(shape, layers, head, k["embed"], k["final_gain"])


def run_forced(m, prompts, steps, seed=0):
    """Teacher-forced run: each sequence b gets prompts[b] (its history), then `steps` forced steps whose tokens come
    from a seeded stream (so the CPU oracle sees the same sequence whatever the GPU chooses). Returns
    (tokens [B][T], gpu_logits [B][steps][V], positions [B] of the logit rows)."""
    rng = np.random.default_rng(seed)
    B = m.batch
    V = m.shape.VOCAB
    seqs = []
    for b in range(B):
        m.start(b, prompts[b])
        seqs.append(list(prompts[b]))
    hist = [len(p) for p in prompts]
    # consume the histories: one step per logged token after the first (positions 0 .. len-2); sequences with
    # shorter prompts are padded with forced tokens so every sequence steps together
    pre = max(hist) - 1
    forced = np.full((pre + steps, B), 0xFFFFFFFF, np.uint64)
    for b in range(B):
        for t in range(hist[b] - 1, pre + steps):
            tok = int(rng.integers(0, V))
            forced[t, b] = tok
            seqs[b].append(tok)
    if pre:
        m.decode(pre, forced=forced[:pre], want_tokens=False)
    toks, lg, _ = m.decode(steps, forced=forced[pre:], want_tokens=True, want_logits=True)
    return seqs, lg, toks


def compare(m, seqs, lg, steps, check_argmax=True, min_margin_factor=4.0, which=None):
    """Per sequence (all, or the indices in `which`): the oracle's logits at the last `steps` positions; returns a
    report dict and asserts the bound and (where the oracle's top-2 margin clears the observed error) the argmax."""
    om = oracle_model(m)
    report = []
    for b in (range(m.batch) if which is None else which):
        toks = seqs[b][: len(seqs[b]) - 1]            # the tokens fed at each position
        T = len(toks)
        pos = list(range(T - steps, T))
        ref64 = om.forward(toks, "fp64", logit_positions=pos)
        refh = om.forward(toks, "half", logit_positions=pos)
        got = lg[:, b, :].astype(np.float64)
        err = np.abs(got - ref64)
        budget = D.logit_bound(ref64)
        assert np.all(np.isfinite(got))
        assert np.all(err <= budget), "logit bound exceeded: max err %.3g, budget fraction %.3g" % (
            err.max(), (err / budget).max())
        eh = np.abs(got - refh).max()
        agree = 0
        for i in range(steps):
            ga, ha = int(np.argmax(got[i])), int(np.argmax(refh[i]))
            margin = D.top2_margin(refh[i])
            if ga == ha:
                agree += 1
            elif check_argmax:
                assert margin <= min_margin_factor * eh, "argmax %d != oracle %d at step %d (margin %.3g, err %.3g)" % (
                    ga, ha, i, margin, eh)
        report.append(dict(max_err_fp64=float(err.max()), budget_frac=float((err / budget).max()),
                           max_err_half=float(eh), argmax_agree=agree, steps=steps))
    return report
