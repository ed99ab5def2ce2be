"""The speculative verify step on the B200 (agxc_model_verify; the reference's verify section, assemble.py:244-253,
747-803): a draft equal to greedy decoding's tokens is accepted whole and the model's next choice follows it; a wrong
draft is cut at its first wrong token and decoding continues from the committed state as greedy decoding would; the
verify rows' logits are within the FP64 oracle's bound; prompt-lookup speculation emits greedy decoding's tokens."""
import numpy as np
import pytest

from oracle import decoder as D
from tests import modelcheck as MC

pytestmark = pytest.mark.gpu

SMALL = dict(NAME="small", D_MODEL=256, LAYERS=2, HEADS=4, KV_HEADS=2, HEAD_DIM=64, FFN=512, VOCAB=1024,
             ROPE_THETA=1e6, EPS=1e-6)


@pytest.fixture(scope="module")
def torch():
    import torch as t
    if not t.cuda.is_available():
        pytest.skip("no GPU")
    return t


def _build(seed=5, cap=128):
    from agxforge.inference import assemble
    m = assemble.build(dict(model=dict(SMALL), bits=4, cap=cap, seed=seed, keep_logits=True), keep_packs=True)
    m.set_option("fused", 0)
    return m


def _greedy(m, image, n):
    m.restore_state(image)
    toks, lg, _ = m.decode(n, want_tokens=True, want_logits=True)
    return [int(t) for t in toks[:, 0]], lg[:, 0, :]


def _clear_margins(lg):
    return min(D.top2_margin(r) for r in lg) > 0.02      # no near-tie the two summation orders could flip


def test_verify_accepts_a_greedy_draft(torch):
    m = _build()
    m.start(0, [3, 14, 15, 92, 65])
    m.decode(4, want_tokens=False)
    image = m.save_state()
    q0 = m.state(0)[0]
    G, glg = _greedy(m, image, 6)
    m.restore_state(image)
    emitted, vlg = m.verify(G[:5], want_logits=True)
    assert np.abs(vlg - glg).max() < 1e-2          # the row pass's logits against the decode step's
    if _clear_margins(glg):
        assert emitted == G[:6]
        assert m.state(0)[0] == q0 + 6
    m.close()


def test_verify_cuts_a_wrong_draft_and_decoding_continues(torch):
    m = _build(seed=6)
    m.start(0, [1, 2, 3, 4, 5, 6])
    m.decode(5, want_tokens=False)
    image = m.save_state()
    q0 = m.state(0)[0]
    G, glg = _greedy(m, image, 8)
    m.restore_state(image)
    wrong = (G[2] + 1) % SMALL["VOCAB"]
    emitted, _ = m.verify(G[:2] + [wrong] + G[3:5])
    if _clear_margins(glg):
        assert emitted == G[:3]
        assert m.state(0)[0] == q0 + 3
        cont, _, _ = m.decode(5, want_tokens=True)
        assert [int(t) for t in cont[:, 0]] == G[3:8]
    m.close()


def test_verify_rows_against_the_oracle(torch):
    m = _build(seed=7)
    rng = np.random.default_rng(7)
    prompt = rng.integers(0, SMALL["VOCAB"], 12).tolist()
    m.start(0, prompt)
    m.decode(len(prompt) - 1, want_tokens=False)    # consume the prompt: q0 = its last position
    draft = rng.integers(0, SMALL["VOCAB"], 7).tolist()
    _, vlg = m.verify(draft, want_logits=True)
    om = MC.oracle_model(m)
    toks = prompt + draft
    pos = list(range(len(prompt) - 1, len(prompt) + len(draft)))
    ref = om.forward(toks, "fp64", logit_positions=pos)
    assert np.all(np.abs(vlg.astype(np.float64) - ref) <= D.logit_bound(ref))
    m.close()


def test_prompt_lookup_generation_equals_greedy(torch):
    from agxforge.inference import speculate
    m = _build(seed=8)
    # a repetitive prompt, so the history offers drafts
    m.start(0, [7, 8, 9, 10, 7, 8, 9, 10, 7, 8, 9, 10])
    m.decode(11, want_tokens=False)
    image = m.save_state()
    G, glg = _greedy(m, image, 24)
    m.restore_state(image)
    out, rounds, drafted, accepted = speculate.generate(m, 24)
    assert len(out) == 24 and rounds <= 24
    if _clear_margins(glg):
        assert out == G
    m.close()
