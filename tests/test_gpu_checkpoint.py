"""Checkpoint import on the B200: an MLX-format checkpoint (two safetensors shards, bf16 scale and bias patterns, wqkv
in the checkpoint's per-KV-group row order, quantized embedding) written by the test, read by
agxforge.inference.checkpoint.load and fed through agxc_model_set_pack. The model built from the file decodes
bit-identically to the model built from the same logical packs directly, and within the FP64 oracle's bound at every
step."""
import numpy as np
import pytest

from agxforge.inference import models
from tests import modelcheck as MC
from tests.test_checkpoint import _mlx_checkpoint

pytestmark = pytest.mark.gpu

SHAPE = models.Model("ckpt", 256, 2, 4, 2, 64, 512, 1024, 1e6, 1e-5)


@pytest.fixture(scope="module")
def torch():
    import torch as t
    if not t.cuda.is_available():
        pytest.skip("no GPU")
    return t


@pytest.mark.parametrize("bits", [4, 8])
def test_checkpoint_model_decodes_like_direct_packs(torch, tmp_path, bits):
    from agxforge.inference import assemble
    from agxforge.inference import checkpoint as CK
    paths, logical = _mlx_checkpoint(str(tmp_path / "m"), SHAPE, bits, seed=bits)
    W, sdt = CK.load(paths, SHAPE, bits)
    cfg = dict(model=SHAPE, bits=bits, scale_dtype=sdt, cap=64, seed=0, keep_logits=True)
    rng = np.random.default_rng(bits)
    prompt = rng.integers(0, SHAPE.VOCAB, 12).tolist()
    out = {}
    for name, weights in (("file", W), ("direct", logical)):
        m = assemble.build(dict(cfg), weights=weights, keep_packs=True)
        m.set_option("fused", 0)            # the per-kernel path sums in a fixed order: bit-comparable
        seqs, lg, _ = MC.run_forced(m, [prompt], 6, seed=3)
        out[name] = lg
        if name == "file":
            m.set_option("fused", 1)
            seqs2, lg2, _ = MC.run_forced(m, [prompt], 6, seed=3)
            MC.compare(m, seqs2, lg2, 6, name="checkpoint q%d fused step" % bits)
        m.close()
    assert np.array_equal(out["file"], out["direct"])
