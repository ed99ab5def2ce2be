"""The reference's per-kernel functions under their own names (agxforge.kernels.*), run on the B200, against the
reference's own values (tests/golden/ref_kernels.npz, made by tests/golden/make_golden.py from the reference's CPU
references), and decode attention against the reference's delivery contract: the true base-2 softmax enclosed within
the row-scaled bound 8.7e-4, with a wrong-base (e^x) control that must land outside it (tools/g17deliver.py:771-793,
802-858: q0 in {0, 5, cap/2, cap-1}, seeds 300 + q0, NaN-poisoned cache rows past the append)."""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATTN_ENCLOSURE_BOUND = 8.7e-4        # the reference's row-scaled softmax enclosure (tools/g17deliver.py:793)
EPS32 = np.finfo(np.float32).eps


@pytest.fixture(scope="module")
def torch():
    import torch as t
    if not t.cuda.is_available():
        pytest.skip("no GPU")
    return t


def _ulp16(x):
    return np.spacing(np.abs(np.asarray(x, np.float64)).astype(np.float16)).astype(np.float64)


@pytest.mark.parametrize("bits", [4, 8])
def test_qmv2_ksplit_reference_by_name(torch, golden, bits):
    from agxforge.kernels import qmv as Q
    from oracle import pack as P
    rp, rs, rb = golden["qmv%d_packed" % bits], golden["qmv%d_s16" % bits], golden["qmv%d_b16" % bits]
    N_, K = rp.shape[0], rp.shape[1] * 32 // bits
    q = P.unpack(rp, bits, N_, K)
    x = golden["qmv%d_x" % bits]
    lay = Q.qmv_layout(N_, K, bits=bits)                 # bf16 scale patterns, as the reference's quantize
    y = Q.qmv2_ksplit_reference(lay, x, q, rs, rb).astype(np.float64)
    W = P.dequant64(q, rs, rb, "bf16")
    bound = 64 * EPS32 * (np.abs(W) @ np.abs(x.astype(np.float64))) + 1e-7
    assert y.shape == (N_,) and np.all(np.abs(y - golden["qmv%d_y" % bits]) <= bound)
    yb = Q.qmv_batch_reference(Q.with_batch(lay, 2), np.stack([x, x]), q, rs, rb)
    assert yb.shape == (2, N_) and np.array_equal(yb[0], yb[1])


def test_qmv_swiglu_reference_by_name(torch, golden):
    from agxforge.kernels import qmv as Q
    from oracle import pack as P
    rp, rs, rb = golden["swiglu_packed"], golden["swiglu_s16"], golden["swiglu_b16"]
    F2, K = rp.shape[0], rp.shape[1] * 8
    lay = Q.qmv_swiglu_layout(F2 // 2, K, bits=4)
    act = Q.qmv_swiglu_reference(lay, golden["swiglu_x"], P.unpack(rp, 4, F2, K), rs, rb)
    want = golden["swiglu_act"].astype(np.float64)
    assert act.dtype == np.float16
    assert np.all(np.abs(act.astype(np.float64) - want) <= 2 * _ulp16(want) + 1e-6)


def test_residual_reference_by_name(torch, golden):
    from agxforge.kernels import qmv as Q
    lay = Q.qmv_layout(256, 256)
    h = Q.residual_reference(Q.with_residual(lay, "add16"), golden["res_y"], x16=golden["res_x16"])
    assert np.array_equal(h.view(np.uint32), golden["res_add16"].view(np.uint32))
    o = Q.residual_reference(Q.with_residual(lay, "add32_to16"), golden["res_y"], h32=golden["res_h32"])
    assert np.array_equal(o.view(np.uint16), golden["res_add32_to16"].view(np.uint16))


def test_rmsnorm_wide_reference_by_name(torch, golden):
    from types import SimpleNamespace

    from agxforge.kernels import norm
    spec = SimpleNamespace(norm_eps=float(golden["norm_eps"]), storage="half")
    for src, want in (("norm_v16", "norm_out16"), ("norm_v32", "norm_out32")):
        y = norm.rmsnorm_wide_reference(golden[src], golden["norm_g"], spec)
        ref = golden[want].astype(np.float64)
        # the reference's rsqrt is correctly rounded; the B200's may differ by one fp32 ulp, which can move the fp16
        # rounding of an element by one ulp
        assert np.all(np.abs(y.astype(np.float64) - ref) <= _ulp16(ref))


def test_argmax_reference_by_name(torch, golden):
    from agxforge.kernels import argmax
    assert argmax.argmax_reference(golden["argmax_logits"]) == int(golden["argmax_index"])   # a tie: first wins
    rng = np.random.default_rng(3)
    for n in (1, 31, 1000, 92544, 151936):
        v = rng.standard_normal(n).astype(np.float32)
        v[rng.integers(0, n, 3)] = v.max()                  # planted ties
        assert argmax.argmax_reference(v) == int(np.argmax(v))


def test_attn_rope_reference_by_name(torch, golden):
    """RoPE + append bit-exact (two rounded products and one rounded sum per element, then fp16), attention output
    within two fp16 ulps of the reference's value."""
    from agxforge.kernels import attention as A
    q0 = int(golden["attn_q0"])
    K, V = golden["attn_K"], golden["attn_V"]
    lay = A.attn_rope_layout(16, 8, 128, cap=K.shape[1])
    out, K2, V2 = A.attn_rope_reference(lay, golden["attn_qkv32"], golden["attn_cos"], golden["attn_sin"], K, V, q0)
    assert np.array_equal(K2[:, q0].view(np.uint16), golden["attn_knew"].view(np.uint16))
    assert np.array_equal(V2[:, q0].view(np.uint16), golden["attn_vnew"].view(np.uint16))
    want = golden["attn_out"].astype(np.float64)
    assert np.all(np.abs(out.astype(np.float64) - want) <= 2 * _ulp16(want) + 1e-3 * np.abs(want).max())


def _true_softmax(q16, K, V, q0, H, KVH, base):
    out = np.zeros((H, q16.shape[1]))
    for h in range(H):
        kv = h // (H // KVH)
        s = K[kv, :q0 + 1].astype(np.float64) @ q16[h].astype(np.float64)
        p = np.exp2(s - s.max()) if base == 2 else np.exp(s - s.max())
        out[h] = (p @ V[kv, :q0 + 1].astype(np.float64)) / p.sum()
    return out


@pytest.mark.parametrize("H,KVH,hd", [(16, 8, 128), (14, 2, 64)])
@pytest.mark.parametrize("q0_at", ["0", "5", "half", "last"])
def test_attention_enclosure_with_wrong_base_control(torch, H, KVH, hd, q0_at):
    """The reference's delivery check of decode attention: inputs as tools/g17deliver.py:802-817 makes them (qkv
    N(0, 1.5^2), RoPE at q0 with theta 1e6, caches N(0, 1) fp16 poisoned with NaN from row q0 on), the device's
    RoPE + append + attention, then (a) the appended K row bit-exact against the restated RoPE, (b) the output within
    8.7e-4 of the true base-2 softmax, row-scaled, and (c) the base-e control outside that bound (except q0 = 0, where
    one key makes every base agree). A kernel with the wrong exponent base fails (b); a check that cannot fail
    fails (c)."""
    from agxforge.kernels import attention as A
    cap = 2048
    q0 = {"0": 0, "5": 5, "half": cap // 2, "last": cap - 1}[q0_at]
    rng = np.random.default_rng(300 + q0)
    qkv = (rng.standard_normal((H + 2 * KVH) * hd) * 1.5).astype(np.float32)
    th = np.float64(1e6) ** (-np.arange(hd // 2) * 2 / hd)
    ang = q0 * th
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    Kc = rng.standard_normal((KVH, cap, hd)).astype(np.float16)
    Vc = rng.standard_normal((KVH, cap, hd)).astype(np.float16)
    Kc[:, q0:] = np.float16(np.nan)
    Vc[:, q0:] = np.float16(np.nan)
    lay = A.attn_rope_layout(H, KVH, hd, cap=cap)
    out, K2, V2 = A.attn_rope_reference(lay, qkv, cos, sin, Kc, Vc, q0)
    # the restated RoPE (numerics.rope_rotate: fp32 products and sum, each rounded; fp16 storage)
    f32 = np.float32
    q = qkv[:H * hd].reshape(H, hd)
    k = qkv[H * hd:(H + KVH) * hd].reshape(KVH, hd)
    v = qkv[(H + KVH) * hd:].reshape(KVH, hd)

    def rot(t):
        h2 = hd // 2
        x1, x2 = t[:, :h2], t[:, h2:]
        return np.concatenate([(x1 * cos).astype(f32) - (x2 * sin).astype(f32),
                               (x2 * cos).astype(f32) + (x1 * sin).astype(f32)], axis=1).astype(f32)

    qs = f32(1.4426950408889634 / math.sqrt(hd))
    q16 = (rot(q) * qs).astype(f32).astype(np.float16)
    k16 = rot(k).astype(np.float16)
    assert np.array_equal(K2[:, q0].view(np.uint16), k16.view(np.uint16))
    assert np.array_equal(V2[:, q0].view(np.uint16), v.astype(np.float16).view(np.uint16))
    Kt, Vt = Kc.copy(), Vc.copy()
    Kt[:, q0], Vt[:, q0] = k16, v.astype(np.float16)
    got = out.astype(np.float64)
    assert np.all(np.isfinite(got))
    true2 = _true_softmax(q16, Kt, Vt, q0, H, KVH, 2)
    truee = _true_softmax(q16, Kt, Vt, q0, H, KVH, "e")
    rowmax = np.abs(true2).max(axis=1, keepdims=True)
    encl = float((np.abs(got - true2) / rowmax).max())
    ctrl = float((np.abs(got - truee) / rowmax).max())
    assert encl <= ATTN_ENCLOSURE_BOUND, encl
    if q0 > 0:
        assert ctrl > ATTN_ENCLOSURE_BOUND, ctrl
