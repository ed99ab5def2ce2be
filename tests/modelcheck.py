"""Shared helpers of the model-level parity tests (test infrastructure): build a device model with its packs kept,
mirror it into the CPU oracle, run a teacher-forced decode on the GPU and compare every step's logits with the FP64
oracle (the reference's bound 0.05 + 0.003*|ref|, tools/g17generationcheck.py:39) and its argmax with the
half-transport oracle's.

The argmax rule (the north star asks for the same top token on every step): the device's token is the first maximum
of its own logits. Where it differs from the half-transport oracle's, the two candidates' half-transport margin must
be within the stated rounding bound oracle.decoder.argmax_rounding_bound (each element of the final normed row one
fp16 ulp off, plus the fp32 dot-product bound); a miss with a larger margin fails. Every step's margin, bound and
agreement is recorded and printed in the session summary (tests/conftest.py)."""
from __future__ import annotations

import time

import numpy as np

from oracle import decoder as D

RECORDS = []          # one dict per compared sequence, printed at the end of the session
_FORWARD = {}         # the last oracle passes, keyed by (model packs, tokens, positions)


def oracle_model(m):
    """The CPU oracle's copy of a DecodeModel built with keep_packs=True."""
    S = m.shape
    shape = D.Shape(S.D_MODEL, S.LAYERS, S.HEADS, S.KV_HEADS, S.HEAD_DIM, S.FFN, S.VOCAB, S.EPS, S.ROPE_THETA,
                    S.QKV_BIAS, S.TIED, S.QK_NORM)
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
        L["qn"] = k.get((l, "q_norm"))
        L["kn"] = k.get((l, "k_norm"))
        layers.append(L)
    head = pack((None, "head"), S.VOCAB, S.D_MODEL)
    return D.Model(shape, layers, head, k["embed"], k["final_gain"])


def run_forced(m, prompts, steps, seed=0, prefill=False):
    """Teacher-forced run: each sequence b gets prompts[b] (its history), then `steps` forced steps whose tokens come
    from a seeded stream (so the CPU oracle sees the same sequence whatever the GPU chooses). The history is consumed
    by forced decode steps (positions 0 .. len-2 one step each) or, with prefill=True, by the prefill section.
    Returns (tokens [B][T], gpu_logits [steps][B][V], device tokens [steps][B])."""
    rng = np.random.default_rng(seed)
    B = m.batch
    V = m.shape.VOCAB
    seqs = [list(p) for p in prompts]
    hist = [len(p) for p in prompts]
    if prefill:
        if len(set(hist)) != 1:
            raise ValueError("run_forced: prefill takes equal-length prompts")
        for b in range(B):
            m.prefill(b, prompts[b])
        pre = 0
        first = hist[0] - 1
    else:
        for b in range(B):
            m.start(b, prompts[b])
        # one step per logged token after the first (positions 0 .. len-2); shorter prompts are padded with forced
        # tokens so every sequence steps together
        pre = max(hist) - 1
        first = None
    forced = np.full((pre + steps, B), 0xFFFFFFFF, np.uint64)
    for b in range(B):
        t0 = hist[b] - 1 if first is None else 0
        for t in range(t0, pre + steps):
            tok = int(rng.integers(0, V))
            forced[t, b] = tok
            seqs[b].append(tok)
    if pre:
        m.decode(pre, forced=forced[:pre], want_tokens=False)
    toks, lg, _ = m.decode(steps, forced=forced[pre:], want_tokens=True, want_logits=True)
    return seqs, lg, toks


def compare(m, seqs, lg, steps, which=None, name="", om=None):
    """Per sequence (all, or the indices in `which`): the oracle's logits at the last `steps` positions. Asserts the
    logit bound at every step and the argmax rule above; returns the per-sequence records."""
    om = om or oracle_model(m)
    report = []
    for b in (range(m.batch) if which is None else which):
        toks = seqs[b][: len(seqs[b]) - 1]            # the tokens fed at each position
        T = len(toks)
        pos = list(range(T - steps, T))
        t0 = time.time()
        key = (id(m.packs), tuple(toks), pos[0], pos[-1])
        if key not in _FORWARD:
            if len(_FORWARD) >= 2:
                _FORWARD.pop(next(iter(_FORWARD)))
            _FORWARD[key] = om.forward_both(toks, pos)
        ref64, refh, xfh, W = _FORWARD[key]
        oracle_s = time.time() - t0
        got = lg[:, b, :].astype(np.float64)
        assert np.all(np.isfinite(got)), "non-finite logits"
        err = np.abs(got - ref64)
        budget = D.logit_bound(ref64)
        eh = np.abs(got - refh).max(axis=1)
        steps_rec = []
        misses = []
        for i in range(steps):
            ga = int(np.argmax(got[i]))
            ha = int(np.argmax(refh[i]))
            margin = D.top2_margin(refh[i])
            rec = dict(step=i, agree=ga == ha, margin=round(margin, 6), err_half=float(eh[i]),
                       budget_frac=float((err[i] / budget[i]).max()))
            if ga != ha:
                gap = float(refh[i][ha] - refh[i][ga])
                bound = D.argmax_rounding_bound(W, xfh[i], ga, ha)
                rec.update(gpu=ga, oracle=ha, gap=gap, bound=bound)
                misses.append(rec)
            steps_rec.append(rec)
        r = dict(name=name, seq=b, positions=[pos[0], pos[-1]], steps=steps, max_err_fp64=float(err.max()),
                 budget_frac=float((err / budget).max()), max_err_half=float(eh.max()),
                 argmax_agree=sum(1 for s in steps_rec if s["agree"]),
                 min_margin=min(s["margin"] for s in steps_rec), misses=misses, oracle_s=round(oracle_s, 1))
        RECORDS.append(r)
        report.append(r)
        assert np.all(err <= budget), "logit bound exceeded: max err %.3g, budget fraction %.3g" % (
            err.max(), (err / budget).max())
        for mrec in misses:
            assert mrec["gap"] <= mrec["bound"], (
                "argmax %d != oracle %d at step %d: half-transport gap %.3g above the rounding bound %.3g" % (
                    mrec["gpu"], mrec["oracle"], mrec["step"], mrec["gap"], mrec["bound"]))
    return report
