"""Full-depth parity of the BASELINE configs on the B200: every layer, the full vocabulary, the BASELINE histories,
every decode step compared.

    config 3   InternLM2.5-1.8B-shaped, 4-bit, 24 layers: histories of 196 and 1,792 tokens reached through the prefill
               section and through forced decode steps, then 64 teacher-forced steps
    config 1   Qwen2.5-0.5B-shaped, 4-bit, 24 layers (qkv bias, tied head): a 196-token prefill, then the BASELINE's
               greedy step and 7 more
    config 4   InternLM2.5-1.8B-shaped, 8-bit: 8 sequences (the GEMV step) and 32 sequences (the tensor-core step), each
               with its own 1,792-token history, then 32 teacher-forced steps; sequences checked against the oracle
               as named per case
    bf16       the config 3 model with reference-format (bf16) scale and bias patterns, 196-token history

Every compared step: logits within 0.05 + 0.003|ref| of the FP64 oracle, and the argmax rule of tests/modelcheck.py
(equal to the half-transport oracle's, or a miss within the stated rounding bound). The records (margins, errors,
agreement) print in the session summary. The oracle is the CPU restatement (oracle/decoder.py), one causal pass per
sequence, both policies together; it takes about a minute per 1,856-position sequence of the 1.8B model."""
import numpy as np
import pytest

from tests import modelcheck as MC

pytestmark = [pytest.mark.gpu, pytest.mark.slow]


@pytest.fixture(scope="module")
def torch():
    import torch as t
    if not t.cuda.is_available():
        pytest.skip("no GPU")
    return t


def _build(model, bits, seed, cap, batch=1, sdt="fp16"):
    from agxforge.inference import assemble
    return assemble.build(dict(model=model, bits=bits, batch=batch, cap=cap, seed=seed, keep_logits=True,
                               scale_dtype=sdt), keep_packs=True)


@pytest.fixture(scope="module")
def internlm_q4(torch):
    m = _build("internlm2.5-1.8b", 4, seed=2, cap=2048)
    yield m
    m.close()


@pytest.mark.parametrize("history", [196, 1792])
@pytest.mark.parametrize("path", ["prefill", "forced"])
def test_config3_full_depth(internlm_q4, history, path):
    m = internlm_q4
    rng = np.random.default_rng(1000 + history)
    prompt = rng.integers(0, m.shape.VOCAB, history).tolist()
    seqs, lg, toks = MC.run_forced(m, [prompt], 64, seed=2000 + history, prefill=path == "prefill")
    # the same token sequence through either path: the oracle's pass is computed once and reused
    MC.compare(m, seqs, lg, 64, name="config3 q4 history %d via %s" % (history, path))
    # then free generation: every token the device chooses is the first maximum of the logits it produced
    free, flg, _ = m.decode(8, want_tokens=True, want_logits=True)
    for i in range(8):
        assert int(free[i, 0]) == int(np.argmax(flg[i, 0]))


def test_config3_full_depth_fused_step(internlm_q4):
    """Config 3 at history 1,792 on the fused persistent step (the same forced sequence as the graph path's case)."""
    m = internlm_q4
    m.set_option("fused", 1)
    try:
        rng = np.random.default_rng(1000 + 1792)
        prompt = rng.integers(0, m.shape.VOCAB, 1792).tolist()
        seqs, lg, toks = MC.run_forced(m, [prompt], 64, seed=2000 + 1792, prefill=False)
        MC.compare(m, seqs, lg, 64, name="config3 q4 history 1792 fused step")
    finally:
        m.set_option("fused", 0)


def test_config1_full_depth(torch):
    m = _build("qwen2.5-0.5b", 4, seed=0, cap=256)
    rng = np.random.default_rng(0)
    prompt = rng.integers(0, m.shape.VOCAB, 196).tolist()
    seqs, lg, toks = MC.run_forced(m, [prompt], 8, seed=1, prefill=True)
    MC.compare(m, seqs, lg, 8, name="config1 qwen q4 prefill 196 + 8 steps")
    m.close()


@pytest.mark.parametrize("batch,which", [(8, [5]), (32, [0, 31])])
def test_config4_q8_full_depth(torch, batch, which):
    m = _build("internlm2.5-1.8b", 8, seed=3, cap=2048, batch=batch)
    rng = np.random.default_rng(3000 + batch)
    prompts = [rng.integers(0, m.shape.VOCAB, 1792).tolist() for _ in range(batch)]
    seqs, lg, toks = MC.run_forced(m, prompts, 32, seed=4000 + batch, prefill=True)
    MC.compare(m, seqs, lg, 32, which=which, name="config4 q8 B%d history 1792" % batch)
    m.close()


def test_bf16_reference_format_full_depth(torch):
    m = _build("internlm2.5-1.8b", 4, seed=5, cap=512, sdt="bf16")
    rng = np.random.default_rng(5)
    prompt = rng.integers(0, m.shape.VOCAB, 196).tolist()
    seqs, lg, toks = MC.run_forced(m, [prompt], 16, seed=6, prefill=True)
    MC.compare(m, seqs, lg, 16, name="config3 shape bf16 packs history 196")
    m.close()
