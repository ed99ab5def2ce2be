"""QK-norm (the Qwen3 family: a per-head RMSNorm of q and k over head_dim, with shared gains, before RoPE;
agxforge/kernels/attention.py:256-265 with_qknorm, tools/g17qwen3.py:216-231) on every decode path — the fused batch-1
step, the per-kernel batch-1..8 path, the tensor-core path for 32 sequences and the prefill section — against the FP64
oracle with the same norm, every step under teacher forcing; and a model without the norm differs (the check can
fail)."""
import numpy as np
import pytest

from tests import modelcheck as MC

pytestmark = pytest.mark.gpu

QK = dict(NAME="qk", D_MODEL=256, LAYERS=2, HEADS=4, KV_HEADS=2, HEAD_DIM=128, FFN=512, VOCAB=1024,
          ROPE_THETA=1e6, EPS=1e-6, QK_NORM=True)


@pytest.fixture(scope="module")
def torch():
    import torch as t
    if not t.cuda.is_available():
        pytest.skip("no GPU")
    return t


def _build(shape, batch=1, cap=96, bits=4, seed=7):
    from agxforge.inference import assemble
    return assemble.build(dict(model=shape, bits=bits, batch=batch, cap=cap, seed=seed, keep_logits=True),
                          keep_packs=True)


@pytest.mark.parametrize("hd", [64, 128])
@pytest.mark.parametrize("fused", [1, 0])
def test_qknorm_batch1(torch, hd, fused):
    m = _build(dict(QK, HEAD_DIM=hd))
    m.set_option("fused", fused)
    rng = np.random.default_rng(hd)
    prompt = rng.integers(0, 1024, 20).tolist()
    seqs, lg, _ = MC.run_forced(m, [prompt], 6, seed=1)
    MC.compare(m, seqs, lg, 6, name="qk-norm hd %d fused %d" % (hd, fused))
    m.close()


def test_qknorm_small_batch_and_prefill(torch):
    m = _build(dict(QK), batch=3)
    rng = np.random.default_rng(3)
    prompts = [rng.integers(0, 1024, 16).tolist() for _ in range(3)]
    seqs, lg, _ = MC.run_forced(m, prompts, 4, seed=2, prefill=True)
    MC.compare(m, seqs, lg, 4, name="qk-norm batch 3 prefill")
    m.close()


def test_qknorm_tensor_core_batch(torch):
    m = _build(dict(QK), batch=32)
    rng = np.random.default_rng(4)
    prompts = [rng.integers(0, 1024, 12).tolist() for _ in range(32)]
    seqs, lg, _ = MC.run_forced(m, prompts, 3, seed=5)
    MC.compare(m, seqs, lg, 3, which=[0, 31], name="qk-norm batch 32")
    m.close()


def test_qwen3_shape_two_layers(torch):
    from agxforge.inference import models
    shape = models.QWEN3_06B.replace(LAYERS=2)
    m = _build(shape, cap=64, seed=11)
    rng = np.random.default_rng(11)
    prompt = rng.integers(0, shape.VOCAB, 24).tolist()
    seqs, lg, _ = MC.run_forced(m, [prompt], 4, seed=12)
    MC.compare(m, seqs, lg, 4, name="qwen3-0.6b shape, 2 layers")
    m.close()


def test_without_the_norm_the_logits_differ(torch):
    """The control: the same packs and gains with QK-norm switched off move the logits far outside the bound."""
    m = _build(dict(QK))
    rng = np.random.default_rng(9)
    prompt = rng.integers(0, 1024, 10).tolist()
    seqs, lg_on, _ = MC.run_forced(m, [prompt], 3, seed=1)
    m.set_option("qk_norm", 0)
    _, lg_off, _ = MC.run_forced(m, [prompt], 3, seed=1)
    assert np.abs(lg_on - lg_off).max() > 0.05
    m.close()
