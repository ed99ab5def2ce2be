"""Decode-state save and restore on the B200 (agxc_model_state_save / _restore): a saved state restored into a fresh
model with the same weights, or into the same model after it decoded on, continues bit for bit as the original
(the per-kernel path sums in a fixed order), and within rounding on the fused step; images of another shape, or
damaged, are refused."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SMALL = dict(NAME="small", D_MODEL=256, LAYERS=2, HEADS=4, KV_HEADS=2, HEAD_DIM=64, FFN=512, VOCAB=1024,
             ROPE_THETA=1e6, EPS=1e-6)


@pytest.fixture(scope="module")
def torch():
    import torch as t
    if not t.cuda.is_available():
        pytest.skip("no GPU")
    return t


def _build(shape=None, seed=0, cap=96, fused=0):
    from agxforge.inference import assemble
    m = assemble.build(dict(model=dict(shape or SMALL), bits=4, cap=cap, seed=seed, keep_logits=True))
    m.set_option("fused", fused)
    return m


@pytest.mark.parametrize("fused", [0, 1])
def test_restore_continues_like_the_original(torch, fused):
    a = _build(fused=fused)
    a.start(0, [11, 22, 33, 44])
    a.decode(10, want_tokens=False)
    image = a.save_state(0)
    t1, l1, _ = a.decode(8, want_tokens=True, want_logits=True)
    # a fresh model with the same weights
    b = _build(fused=fused)
    b.restore_state(image, 0)
    t2, l2, _ = b.decode(8, want_tokens=True, want_logits=True)
    # the same model, rewound
    a.restore_state(image, 0)
    t3, l3, _ = a.decode(8, want_tokens=True, want_logits=True)
    # a fresh model with a larger cache (its attention may split the keys differently: equal to rounding)
    c = _build(fused=fused, cap=128)
    c.restore_state(image, 0)
    t4, l4, _ = c.decode(8, want_tokens=True, want_logits=True)
    assert np.abs(l1 - l4).max() < 1e-3
    if fused:   # float atomics: the order of the split-K sums varies, the values agree to rounding
        assert np.abs(l1 - l2).max() < 1e-3 and np.abs(l1 - l3).max() < 1e-3
    else:
        assert np.array_equal(t1, t2) and np.array_equal(t1, t3)
        assert np.array_equal(l1, l2) and np.array_equal(l1, l3)
    for m in (b, c):   # start() logs the prompt for teacher forcing at q0 = 0: 10 + 8 steps since
        q0, log = m.state(0)
        assert q0 == 10 + 8
        assert list(log[:4]) == [11, 22, 33, 44]
    for m in (a, b, c):
        m.close()


def test_restore_refuses_mismatches(torch):
    a = _build()
    a.start(0, [1, 2, 3])
    a.decode(10, want_tokens=False)   # q0 = 10: past a 6-row cache
    image = a.save_state(0)
    other = _build(dict(SMALL, LAYERS=3))
    with pytest.raises(ValueError, match="shapes"):
        other.restore_state(image, 0)
    with pytest.raises(ValueError):
        a.restore_state(b"XXXX" + image[4:], 0)
    with pytest.raises(ValueError):
        a.restore_state(image[:-2], 0)
    small_cap = _build(cap=6)
    with pytest.raises(ValueError, match="cap"):
        small_cap.restore_state(image, 0)
    for m in (a, other, small_cap):
        m.close()
