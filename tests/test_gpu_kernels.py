"""Kernel-level parity on the B200: every CUDA kernel against the CPU oracle on the same seeded inputs.

    quantize / unpack / dequant     bit-exact (the reference's quantize and dequant contract)
    GEMV (4 and 8 bits, 1..8 rows)  against the FP64 GEMV of the same pack: |err| <= 32 eps32 sum|w x| (+ one fp16
                                    ulp per staged x element when the RMSNorm prologue rounds x)
    epilogues                       add16, add32_to16, SwiGLU against FP64 with their fp16 output rounding
    attention                       against the FP64 base-2 softmax; cache rows past q0 are NaN-poisoned
                                    (the reference's attention.case, attention.py:1688-1698), so a read of them fails
    rmsnorm                         within one fp16 ulp of the FP64 norm
"""
import numpy as np
import pytest

from oracle import decoder as D
from oracle import pack as P

pytestmark = pytest.mark.gpu

EPS32 = np.finfo(np.float32).eps


@pytest.fixture(scope="module")
def torch():
    import torch as t
    if not t.cuda.is_available():
        pytest.skip("no GPU")
    return t


def _w(rng, n, k, std=0.02):
    return (rng.standard_normal((n, k)) * std).astype(np.float32)


def ulp16(v):
    return np.spacing(np.abs(np.asarray(v, np.float64)).astype(np.float16)).astype(np.float64)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("sdt", ["fp16", "bf16"])
def test_quantize_bit_exact(torch, bits, sdt):
    from agxforge.kernels import qmv as Q
    rng = np.random.default_rng(100 + bits)
    W = _w(rng, 96, 512)
    W[1, :64] = 0.25                                   # constant group
    W[2, 64:128] *= 40                                 # wide group
    packed, s16, b16, q = Q.quantize(W, bits=bits, scale_dtype=sdt)
    rp, rs, rb, rq = P.quantize(W, bits=bits, scale_dtype=sdt)
    assert np.array_equal(s16, rs)
    assert np.array_equal(b16, rb)
    assert np.array_equal(packed, rp)
    assert q.dtype == np.uint32 and np.array_equal(q, rq.astype(np.uint32))


@pytest.mark.parametrize("bits", [4, 8])
def test_quantize_matches_reference_golden(torch, golden, bits):
    from agxforge.kernels import qmv as Q
    packed, s16, b16, q = Q.quantize(golden["quant%d_W" % bits], bits=bits)   # bf16, the reference's default
    assert np.array_equal(q, golden["quant%d_q" % bits].astype(np.uint32))
    assert np.array_equal(packed, golden["quant%d_packed" % bits])
    assert np.array_equal(s16, golden["quant%d_s16" % bits])
    assert np.array_equal(b16, golden["quant%d_b16" % bits])


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("sdt", ["fp16", "bf16"])
def test_unpack_dequant_bit_exact(torch, bits, sdt):
    from agxforge.kernels import qmv as Q
    rng = np.random.default_rng(7)
    W = _w(rng, 48, 320)
    rp, rs, rb, rq = P.quantize(W, bits=bits, scale_dtype=sdt)
    pk = Q.Pack(rp, rs, rb, 48, 320, bits=bits, scale_dtype=sdt)
    assert np.array_equal(pk.unpack().cpu().numpy(), rq.astype(np.uint8))
    w = pk.dequant().cpu().numpy()
    assert np.array_equal(w.view(np.uint32), P.dequant(rq, rs, rb, sdt).view(np.uint32))


def test_gateup_pack_layout_bit_exact(torch):
    from agxforge.kernels import qmv as Q
    rng = np.random.default_rng(8)
    Wg, Wu = _w(rng, 64, 256), _w(rng, 64, 256)
    g = P.quantize(Wg, 4, scale_dtype="fp16")
    u = P.quantize(Wu, 4, scale_dtype="fp16")
    pk = Q.Pack.gateup(g[:3], u[:3], 64, 256, bits=4)
    q = pk.unpack().cpu().numpy()
    assert np.array_equal(q[:64], g[3]) and np.array_equal(q[64:], u[3])


def _gemv_case(torch, bits, N_, K, nb, sdt="fp16", seed=0):
    from agxforge.kernels import qmv as Q
    rng = np.random.default_rng(seed)
    W = _w(rng, N_, K)
    rp, rs, rb, rq = P.quantize(W, bits=bits, scale_dtype=sdt)
    pk = Q.Pack(rp, rs, rb, N_, K, bits=bits, scale_dtype=sdt)
    x16 = rng.standard_normal((nb, K)).astype(np.float16)
    W64 = P.dequant64(rq, rs, rb, sdt)
    return pk, x16, W64


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("shape", [(16, 64), (64, 1024), (4096, 2048), (2048, 8192), (1152, 896), (896, 4864)])
@pytest.mark.parametrize("nb", [1, 3, 8])
def test_gemv_f32(torch, bits, shape, nb):
    from agxforge.kernels import qmv as Q
    N_, K = shape
    pk, x16, W64 = _gemv_case(torch, bits, N_, K, nb, seed=N_ + K + nb)
    y = Q.qmv(pk, torch.from_numpy(x16).cuda()).cpu().numpy().astype(np.float64)
    x = x16.astype(np.float64)
    ref = x @ W64.T
    bound = 32 * EPS32 * (np.abs(x) @ np.abs(W64).T) + 1e-7
    err = np.abs(y - ref)
    assert np.all(err <= bound), (err.max(), bound[err > bound][:4])


@pytest.mark.parametrize("splits", [1, 2, 4, 8, 32])
def test_gemv_splits_agree(torch, splits):
    from agxforge.kernels import qmv as Q
    pk, x16, W64 = _gemv_case(torch, 4, 256, 2048, 2, seed=3)
    y = Q.qmv(pk, torch.from_numpy(x16).cuda(), splits=splits).cpu().numpy().astype(np.float64)
    ref = x16.astype(np.float64) @ W64.T
    bound = 32 * EPS32 * (np.abs(x16.astype(np.float64)) @ np.abs(W64).T) + 1e-7
    assert np.all(np.abs(y - ref) <= bound)


def test_gemv_bf16_scales(torch):
    from agxforge.kernels import qmv as Q
    pk, x16, W64 = _gemv_case(torch, 4, 512, 1024, 1, sdt="bf16", seed=5)
    y = Q.qmv(pk, torch.from_numpy(x16).cuda()).cpu().numpy().astype(np.float64)
    ref = x16.astype(np.float64) @ W64.T
    assert np.all(np.abs(y - ref) <= 32 * EPS32 * (np.abs(x16.astype(np.float64)) @ np.abs(W64).T) + 1e-7)


def test_gemv_matches_reference_kernel_golden(torch, golden):
    """The reference's own qmv2_ksplit_reference values (bf16 packs, fp16-valued x) within fp32 rounding."""
    from agxforge.kernels import qmv as Q
    for bits in (4, 8):
        rp, rs, rb = golden["qmv%d_packed" % bits], golden["qmv%d_s16" % bits], golden["qmv%d_b16" % bits]
        N_, K = rp.shape[0], rp.shape[1] * 32 // bits
        pk = Q.Pack(rp, rs, rb, N_, K, bits=bits, scale_dtype="bf16")
        x = golden["qmv%d_x" % bits]
        y = Q.qmv(pk, torch.from_numpy(x.astype(np.float16)).cuda()).cpu().numpy()[0].astype(np.float64)
        W = P.dequant64(P.unpack(rp, bits, N_, K), rs, rb, "bf16")
        bound = 64 * EPS32 * (np.abs(W) @ np.abs(x.astype(np.float64))) + 1e-7
        assert np.all(np.abs(y - golden["qmv%d_y" % bits]) <= bound)


@pytest.mark.parametrize("x_f32", [False, True])
def test_gemv_norm_prologue(torch, x_f32):
    from agxforge.kernels import qmv as Q
    rng = np.random.default_rng(11)
    N_, K, nb = 1024, 2048, 2
    pk, _, W64 = _gemv_case(torch, 4, N_, K, nb, seed=11)
    v = (rng.standard_normal((nb, K)) * 3).astype(np.float32 if x_f32 else np.float16)
    g = (1 + 0.1 * rng.standard_normal(K)).astype(np.float16)
    eps = 1e-5
    y = Q.qmv(pk, torch.from_numpy(v).cuda(), norm_gain=torch.from_numpy(g).cuda(), eps=eps)
    y = y.cpu().numpy().astype(np.float64)
    xr = D.rmsnorm(v.astype(np.float64), g.astype(np.float64), eps, half=True)
    ref = xr @ W64.T
    # the staged row may differ from the FP64 norm's fp16 rounding by one fp16 ulp per element (fp32 rsqrt)
    bound = (ulp16(xr) @ np.abs(W64).T) + 32 * EPS32 * (np.abs(xr) @ np.abs(W64).T) + 1e-7
    assert np.all(np.abs(y - ref) <= bound)


def test_residual_epilogues(torch):
    from agxforge.kernels import qmv as Q
    rng = np.random.default_rng(12)
    pk, x16, W64 = _gemv_case(torch, 4, 512, 1024, 2, seed=12)
    ref = x16.astype(np.float64) @ W64.T
    bound = 32 * EPS32 * (np.abs(x16.astype(np.float64)) @ np.abs(W64).T) + 1e-7
    r16 = rng.standard_normal((2, 512)).astype(np.float16)
    h = Q.qmv(pk, torch.from_numpy(x16).cuda(), epi="add16", res=torch.from_numpy(r16).cuda()).cpu().numpy()
    assert h.dtype == np.float32
    assert np.all(np.abs(h - (ref + r16)) <= bound + np.abs(ref + r16) * EPS32)
    r32 = rng.standard_normal((2, 512)).astype(np.float32)
    o = Q.qmv(pk, torch.from_numpy(x16).cuda(), epi="add32_to16", res=torch.from_numpy(r32).cuda()).cpu().numpy()
    assert o.dtype == np.float16
    want = ref + r32
    assert np.all(np.abs(o.astype(np.float64) - want) <= bound + ulp16(want))


def test_swiglu_epilogue(torch):
    from agxforge.kernels import qmv as Q
    rng = np.random.default_rng(13)
    F, K, nb = 512, 1024, 3
    Wg, Wu = _w(rng, F, K), _w(rng, F, K)
    g = P.quantize(Wg, 4, scale_dtype="fp16")
    u = P.quantize(Wu, 4, scale_dtype="fp16")
    pk = Q.Pack.gateup(g[:3], u[:3], F, K, bits=4)
    x16 = rng.standard_normal((nb, K)).astype(np.float16)
    act = Q.qmv(pk, torch.from_numpy(x16).cuda(), epi="swiglu").cpu().numpy().astype(np.float64)
    x = x16.astype(np.float64)
    G64 = P.dequant64(g[3], g[1], g[2], "fp16")
    U64 = P.dequant64(u[3], u[1], u[2], "fp16")
    gv, uv = x @ G64.T, x @ U64.T
    want = D.silu(gv) * uv
    eg = 32 * EPS32 * (np.abs(x) @ np.abs(G64).T)
    eu = 32 * EPS32 * (np.abs(x) @ np.abs(U64).T)
    bound = np.abs(uv) * eg * 1.2 + np.abs(D.silu(gv)) * eu + ulp16(want) + 1e-6 * np.abs(want)
    assert np.all(np.abs(act - want) <= bound)


def test_rmsnorm_standalone(torch):
    from agxforge.kernels import norm
    rng = np.random.default_rng(14)
    v = (rng.standard_normal((3, 2048)) * 2).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(2048)).astype(np.float16)
    y = norm.rmsnorm(torch.from_numpy(v).cuda(), torch.from_numpy(g).cuda(), 1e-5).cpu().numpy()
    ref = D.rmsnorm(v.astype(np.float64), g.astype(np.float64), 1e-5, half=False)
    assert np.all(np.abs(y.astype(np.float64) - ref) <= ulp16(ref))


@pytest.mark.parametrize("H,KVH,hd", [(16, 8, 128), (14, 2, 64), (32, 8, 128), (4, 4, 64)])
@pytest.mark.parametrize("q0", [0, 5, 196, 1791])
def test_attention(torch, H, KVH, hd, q0):
    from agxforge.kernels import attention as A
    rng = np.random.default_rng(300 + q0)
    cap = 2048
    nb = 2
    q16 = (rng.standard_normal((nb, H, hd)) * 2.0 * (1.4426950408889634 / np.sqrt(hd))).astype(np.float16)
    K = rng.standard_normal((nb, KVH, cap, hd)).astype(np.float16)
    V = rng.standard_normal((nb, KVH, cap, hd)).astype(np.float16)
    q0s = np.array([q0, max(0, q0 - 3)], np.int32)
    for b in range(nb):
        K[b, :, q0s[b] + 1:] = np.float16(np.nan)          # poison: a read past q0 turns the output NaN
        V[b, :, q0s[b] + 1:] = np.float16(np.nan)
    out = A.attention(torch.from_numpy(q16).cuda(), torch.from_numpy(K).cuda(), torch.from_numpy(V).cuda(),
                      q0s).cpu().numpy().astype(np.float64).reshape(nb, H, hd)
    assert np.all(np.isfinite(out))
    for b in range(nb):
        ref = D.attention_step(q16[b].astype(np.float64), K[b], V[b], int(q0s[b]) + 1, KVH)
        # the reference's row-scaled enclosure of the true base-2 softmax (tools/g17deliver.py:793)
        rowmax = np.abs(ref).max(axis=1, keepdims=True)
        assert (np.abs(out[b] - ref) / rowmax).max() <= 8.7e-4


def test_attention_splits_agree(torch):
    from agxforge.kernels import attention as A
    rng = np.random.default_rng(9)
    H, KVH, hd, cap, q0 = 16, 8, 128, 1024, 900
    q16 = (rng.standard_normal((1, H, hd)) * 0.25).astype(np.float16)
    K = rng.standard_normal((1, KVH, cap, hd)).astype(np.float16)
    V = rng.standard_normal((1, KVH, cap, hd)).astype(np.float16)
    ref = D.attention_step(q16[0].astype(np.float64), K[0], V[0], q0 + 1, KVH)
    for S in (1, 2, 4, 8, 16):
        out = A.attention(torch.from_numpy(q16).cuda(), torch.from_numpy(K).cuda(), torch.from_numpy(V).cuda(),
                          [q0], splits=S).cpu().numpy().astype(np.float64).reshape(H, hd)
        rowmax = np.abs(ref).max(axis=1, keepdims=True)
        assert (np.abs(out - ref) / rowmax).max() <= 8.7e-4


def test_bad_shapes_raise(torch):
    from agxforge.kernels import qmv as Q
    with pytest.raises(ValueError):
        Q.Pack(np.zeros((10, 8), np.uint32), np.zeros((10, 1), np.uint16), np.zeros((10, 1), np.uint16), 10, 64)
    rng = np.random.default_rng(1)
    pk, x16, _ = _gemv_case(torch, 4, 64, 256, 1)
    with pytest.raises(ValueError):
        Q.qmv(pk, torch.zeros((1, 128), dtype=torch.float16, device="cuda"))
    with pytest.raises(ValueError):
        Q.qmv(pk, torch.zeros((9, 256), dtype=torch.float16, device="cuda"))


@pytest.mark.parametrize("rw,cg,st", [(1, 32, 2), (2, 16, 3), (4, 8, 4), (8, 4, 8), (8, 16, 2), (1, 2, 5)])
@pytest.mark.parametrize("nb", [1, 3])
def test_gemv_plan_overrides_agree(torch, rw, cg, st, nb):
    """Every unit shape (row tiles x K lanes), chunk size and ring depth computes the same GEMV."""
    from agxforge.kernels import qmv as Q
    pk, x16, W64 = _gemv_case(torch, 4, 512, 2048, nb, seed=21)
    y = Q.qmv(pk, torch.from_numpy(x16).cuda(), row_tiles=rw, chunk_groups=cg, stages=st).cpu().numpy()
    ref = x16.astype(np.float64) @ W64.T
    bound = 32 * EPS32 * (np.abs(x16.astype(np.float64)) @ np.abs(W64).T) + 1e-7
    assert np.all(np.abs(y.astype(np.float64) - ref) <= bound)


@pytest.mark.parametrize("rw", [2, 4, 8])
def test_swiglu_unit_shapes(torch, rw):
    from agxforge.kernels import qmv as Q
    rng = np.random.default_rng(31)
    F, K = 256, 1024
    g = P.quantize(_w(rng, F, K), 4, scale_dtype="fp16")
    u = P.quantize(_w(rng, F, K), 4, scale_dtype="fp16")
    pk = Q.Pack.gateup(g[:3], u[:3], F, K, bits=4)
    x16 = rng.standard_normal((1, K)).astype(np.float16)
    act = Q.qmv(pk, torch.from_numpy(x16).cuda(), epi="swiglu", row_tiles=rw).cpu().numpy().astype(np.float64)
    x = x16.astype(np.float64)
    gv = x @ P.dequant64(g[3], g[1], g[2], "fp16").T
    uv = x @ P.dequant64(u[3], u[1], u[2], "fp16").T
    want = D.silu(gv) * uv
    assert np.all(np.abs(act - want) <= 2 * ulp16(want) + 1e-4 * np.abs(want).max())
