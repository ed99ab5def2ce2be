"""The prefill section on the B200 (agxc_model_prefill): the prompt as chunks of up to 256 rows through the
tensor-core GEMMs and the causal prefill attention, then decode. Checked under teacher forcing against the FP64
oracle (bound 0.05 + 0.003|ref|) and the half-transport argmax, the KV cache rows it wrote against the oracle's, and
the logits against the same prompt fed through decode steps."""
import numpy as np
import pytest

from tests import modelcheck as MC

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as t
    if not t.cuda.is_available():
        pytest.skip("no GPU")
    return t


SMALL = dict(NAME="small", D_MODEL=256, LAYERS=2, HEADS=4, KV_HEADS=2, HEAD_DIM=64, FFN=512, VOCAB=1024,
             ROPE_THETA=1e6, EPS=1e-6)


def _build(shape, bits=4, batch=1, cap=320, seed=0):
    from agxforge.inference import assemble
    return assemble.build(dict(model=shape, bits=bits, batch=batch, cap=cap, seed=seed, keep_logits=True),
                          keep_packs=True)


def _prefill_then_forced(m, b_prompts, steps, seed):
    """prefill every sequence's prompt (equal lengths), then `steps` forced decode steps; the MC.compare inputs."""
    rng = np.random.default_rng(seed)
    V = m.shape.VOCAB
    seqs, forced, info = [], np.zeros((steps, m.batch), np.int64), None
    for b, p in enumerate(b_prompts):
        info = m.prefill(b, p)
        f = rng.integers(0, V, steps)
        forced[:, b] = f
        seqs.append(list(p) + [int(x) for x in f])
    _, lg, _ = m.decode(steps, forced=forced, want_tokens=True, want_logits=True)
    return seqs, lg, info


@pytest.mark.parametrize("bits", [4, 8])
def test_prefill_small_against_oracle_and_decode_path(torch, bits):
    m = _build(dict(SMALL, QKV_BIAS=True), bits=bits, seed=1)
    prompt = np.random.default_rng(2).integers(0, 1024, 300).tolist()     # two chunks: 256 + 43 rows
    seqs, lg, info = _prefill_then_forced(m, [prompt], 4, seed=3)
    MC.compare(m, seqs, lg, 4)
    q0, log = m.state(0)
    assert q0 == len(seqs[0]) - 1 and list(log[:len(seqs[0])]) == seqs[0]
    # the same prompt fed through 299 decode steps: the same logits within a small rounding difference
    m.start(0, prompt)
    m.decode(len(prompt) - 1, want_tokens=False)
    f = np.array(seqs[0][len(prompt):], np.int64).reshape(-1, 1)
    _, lg2, _ = m.decode(4, forced=f, want_tokens=True, want_logits=True)
    assert np.abs(lg2.astype(np.float64) - lg).max() < 0.02
    m.close()


def test_prefill_cache_rows_match_oracle(torch):
    m = _build(dict(SMALL), bits=4, seed=4)
    prompt = np.random.default_rng(5).integers(0, 1024, 70).tolist()
    m.prefill(0, prompt)
    T = len(prompt) - 1
    om = MC.oracle_model(m)
    _, kept = om.forward(prompt[:T], "half", keep=True)
    for l in range(m.shape.LAYERS):
        k, v = m.read_kv(l, 0, T)
        kr, vr = kept[l]
        kr, vr = kr.transpose(1, 0, 2), vr.transpose(1, 0, 2)
        ulp_k = np.spacing(np.abs(kr).astype(np.float16)).astype(np.float64)
        ulp_v = np.spacing(np.abs(vr).astype(np.float16)).astype(np.float64)
        assert np.all(np.abs(k.astype(np.float64) - kr) <= 8 * ulp_k + 1e-2 * np.abs(kr).max())
        assert np.all(np.abs(v.astype(np.float64) - vr) <= 8 * ulp_v + 1e-2 * np.abs(vr).max())
    m.close()


@pytest.mark.parametrize("name,bits,plen", [("internlm2.5-1.8b", 4, 600), ("qwen2.5-0.5b", 4, 150)])
def test_prefill_baseline_shapes_two_layers(torch, name, bits, plen):
    from agxforge.inference import models
    shape = models.get(name).replace(LAYERS=2)
    m = _build(shape, bits=bits, cap=plen + 16, seed=6)
    prompt = np.random.default_rng(7).integers(0, shape.VOCAB, plen).tolist()
    seqs, lg, info = _prefill_then_forced(m, [prompt], 2, seed=8)
    MC.compare(m, seqs, lg, 2)
    assert info["gpu_ms"] > 0
    m.close()


def test_prefill_in_a_batched_model(torch):
    """One sequence of a 32-sequence model (tensor-core decode step) prefilled, the others started token by token."""
    m = _build(dict(SMALL), bits=4, batch=32, cap=160, seed=9)
    rng = np.random.default_rng(10)
    prompts = [rng.integers(0, 1024, 100).tolist() for _ in range(32)]
    for b in range(32):
        if b == 5:
            m.prefill(b, prompts[b])
        else:
            m.start(b, prompts[b])
    m.decode(10, want_tokens=False)   # the others consume their prompts; sequence 5 decodes on from position 99
    assert m.state(5)[0] == 109 and m.state(0)[0] == 10
    m.close()
    # sequence 5 alone: prefill then forced steps, against the oracle
    m = _build(dict(SMALL), bits=4, batch=32, cap=160, seed=9)
    for b in range(32):
        m.prefill(b, prompts[b])
    f = rng.integers(0, 1024, (3, 32))
    _, lg, _ = m.decode(3, forced=f, want_tokens=True, want_logits=True)
    seqs = [prompts[b] + [int(x) for x in f[:, b]] for b in range(32)]
    MC.compare(m, seqs, lg, 3, which=[0, 5, 31])
    m.close()
