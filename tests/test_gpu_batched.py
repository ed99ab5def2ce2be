"""The batched decode step (32..256 sequences: RMSNorm, the tcgen05 GEMM of qmm.cu for every projection and the
vocabulary head, per-row RoPE/append, residual, SwiGLU and argmax kernels, the split-KV attention) on the B200,
under teacher forcing: every checked sequence's logits against the FP64 oracle (bound 0.05 + 0.003*|ref|), its
argmax against the half-transport oracle, and its token log and KV cache rows; free generation picks the first
argmax of the logits it produced."""
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


def _build(shape, bits=4, batch=32, cap=64, seed=0):
    from agxforge.inference import assemble
    return assemble.build(dict(model=shape, bits=bits, batch=batch, cap=cap, seed=seed, keep_logits=True),
                          keep_packs=True)


@pytest.mark.parametrize("bits,batch", [(4, 32), (8, 32), (4, 48)])
def test_batched_small_forced_decode(torch, bits, batch):
    m = _build(dict(SMALL, QKV_BIAS=True), bits=bits, batch=batch)
    rng = np.random.default_rng(11)
    prompts = [rng.integers(0, 1024, int(n)).tolist() for n in rng.integers(3, 24, batch)]
    seqs, lg, toks = MC.run_forced(m, prompts, 4, seed=12)
    which = [0, 1, batch // 2, batch - 1]
    MC.compare(m, seqs, lg, 4, which=which)
    for b in which:  # the token log and position of every checked sequence
        q0, log = m.state(b)
        T = len(seqs[b])
        assert q0 == T - 1
        assert list(log[:T]) == seqs[b]
    m.close()


def test_batched_matches_single_sequence_model(torch):
    """Sequence 7 of a 32-sequence model (tensor-core GEMM step) and the same tokens on a batch-1 model (GEMV step,
    same weights): the logits agree to well inside the oracle bound."""
    from agxforge.inference import assemble
    m = _build(dict(SMALL), bits=4, batch=32, seed=5)
    rng = np.random.default_rng(13)
    prompts = [rng.integers(0, 1024, 10).tolist() for _ in range(32)]
    seqs, lg, _ = MC.run_forced(m, prompts, 3, seed=14)
    # the same seed generates the same weights on the device
    m1 = assemble.build(dict(model=dict(SMALL), bits=4, batch=1, cap=64, seed=5, keep_logits=True))
    m1.start(0, prompts[7])
    forced = np.array(seqs[7][len(prompts[7]):], np.int64).reshape(-1, 1)
    m1.decode(len(prompts[7]) - 1, want_tokens=False)  # the logged prompt
    _, lg1, _ = m1.decode(3, forced=forced, want_tokens=True, want_logits=True)
    d = np.abs(lg[:, 7, :].astype(np.float64) - lg1[:, 0, :])
    assert d.max() < 0.05, "batched vs single-sequence logits differ by %.3g" % d.max()
    m.close()
    m1.close()


def test_batched_free_generation_argmax_is_device_argmax(torch):
    m = _build(dict(SMALL), bits=4, batch=32, seed=2)
    for b in range(32):
        m.start(b, [(5 * b + 1) % 1024, (17 * b + 3) % 1024, 33])
    m.decode(2, want_tokens=False)
    toks, lg, _ = m.decode(5, want_tokens=True, want_logits=True)
    for i in range(5):
        for b in range(32):
            assert int(toks[i, b]) == int(np.argmax(lg[i, b]))
    q0, log = m.state(9)
    assert q0 == 7
    assert list(log[3:8]) == [int(t) for t in toks[:, 9]]
    m.close()


@pytest.mark.parametrize("bits", [4, 8])
def test_batched_internlm_shape_two_layers(torch, bits):
    from agxforge.inference import models
    shape = models.INTERNLM25_18B.replace(LAYERS=2)
    m = _build(shape, bits=bits, batch=32, cap=160, seed=6)
    rng = np.random.default_rng(15)
    prompts = [rng.integers(0, shape.VOCAB, int(n)).tolist() for n in rng.integers(20, 140, 32)]
    seqs, lg, _ = MC.run_forced(m, prompts, 2, seed=16)
    MC.compare(m, seqs, lg, 2, which=[0, 31])
    m.close()


def test_batched_plan_rejects_unaligned_shapes(torch):
    from agxforge.inference import assemble
    with pytest.raises(ValueError):
        assemble.configure(dict(model=dict(SMALL), batch=20))
    with pytest.raises(Exception, match="multiples of 128"):  # vocab 1040: 16-row tiles, not 128-row GEMM tiles
        assemble.build(dict(model=dict(SMALL, VOCAB=1040), bits=4, batch=32, cap=64, seed=0))
    assemble.build(dict(model=dict(SMALL, VOCAB=1040), bits=4, batch=8, cap=64, seed=0)).close()


def test_batched_step_is_deterministic(torch):
    """The split-K GEMMs add their K ranges in a fixed order (no atomics on the data): two runs of the same forced
    decode give bit-identical logits."""
    outs = []
    for _ in range(2):
        m = _build(dict(SMALL), bits=4, batch=32, seed=12)
        rng = np.random.default_rng(13)
        for b in range(32):
            m.start(b, rng.integers(0, 1024, 6).tolist())
        m.decode(5, want_tokens=False)
        f = rng.integers(0, 1024, (3, 32))
        _, lg, _ = m.decode(3, forced=f, want_tokens=True, want_logits=True)
        outs.append(lg)
        m.close()
    assert np.array_equal(outs[0], outs[1])
