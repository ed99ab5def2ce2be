"""Pin the CPU oracle against the reference's own kernel references (tests/golden/ref_kernels.npz).

Pack, unpack and dequant must be bit-exact; the FP64 GEMV/norm/attention restatements must agree with the reference's
fp32-ordered values within the fp32 rounding those orders introduce (the reference's values are single-precision
chains; the oracle is float64 with rounding only at fp16 storage points).
"""
import numpy as np

from oracle import decoder as D
from oracle import pack as P


def test_quantize_bit_exact(golden):
    for bits in (4, 8):
        W = golden["quant%d_W" % bits]
        packed, s16, b16, q = P.quantize(W, bits=bits, scale_dtype="bf16")
        assert np.array_equal(packed, golden["quant%d_packed" % bits])
        assert np.array_equal(s16, golden["quant%d_s16" % bits])
        assert np.array_equal(b16, golden["quant%d_b16" % bits])
        assert np.array_equal(q.astype(np.uint8), golden["quant%d_q" % bits])


def test_unpack_pack_roundtrip(golden):
    for bits in (4, 8):
        packed, q = golden["quant%d_packed" % bits], golden["quant%d_q" % bits]
        N, K = q.shape
        assert np.array_equal(P.unpack(packed, bits, N, K), q)
        assert np.array_equal(P.pack(q, bits), packed)


def test_dequant_bit_exact(golden):
    for bits in (4, 8):
        w = P.dequant(golden["quant%d_q" % bits], golden["quant%d_s16" % bits], golden["quant%d_b16" % bits], "bf16")
        assert w.dtype == np.float32
        assert np.array_equal(w.view(np.uint32), golden["quant%d_wdq" % bits].view(np.uint32))


def test_constant_group_edge(golden):
    # a constant group quantises to scale 1.0 and fields 0 (qmv.py:1864), and dequantises to the constant
    s = P.from_bf16(golden["quant4_s16"])
    assert s[3, 0] == 1.0
    assert np.all(golden["quant4_q"][3, :64] == 0)


def _pack(golden, name, bits):
    packed = golden[name + "_packed"]
    N = packed.shape[0]
    K = packed.shape[1] * 32 // bits
    return D.Pack(packed, golden[name + "_s16"], golden[name + "_b16"], bits, "bf16", N, K)


def test_gemv_matches_reference_order(golden):
    for bits in (4, 8):
        pk = _pack(golden, "qmv%d" % bits, bits)
        x = golden["qmv%d_x" % bits].astype(np.float64)
        W = pk.w64()
        y64 = W @ x
        yref = golden["qmv%d_y" % bits].astype(np.float64)
        # fp32 chains over K=1024 terms: bound by a few ulps of sum |w x|
        bound = 8 * np.finfo(np.float32).eps * (np.abs(W) @ np.abs(x)) + 1e-7
        assert np.all(np.abs(y64 - yref) <= bound)


def test_swiglu_matches_reference(golden):
    pk = _pack(golden, "swiglu", 4)
    F = pk.N // 2
    y = pk.w64() @ golden["swiglu_x"].astype(np.float64)
    act = D.f16(D.silu(y[:F]) * y[F:])
    ref = golden["swiglu_act"].astype(np.float64)
    # fp16 outputs: within one fp16 ulp of the reference's (its exp2_soft SiLU and fp32 chain may round the other way)
    ulp = np.spacing(np.abs(ref).astype(np.float16)).astype(np.float64)
    assert np.all(np.abs(act - ref) <= ulp + 1e-7)


def test_residual_epilogues(golden):
    y, x16, h32 = golden["res_y"], golden["res_x16"], golden["res_h32"]
    assert np.array_equal((y + x16.astype(np.float32)).astype(np.float32), golden["res_add16"])
    assert np.array_equal((y + h32).astype(np.float32).astype(np.float16), golden["res_add32_to16"])


def test_rmsnorm_matches_reference(golden):
    eps = float(golden["norm_eps"])
    for src, ref in (("norm_v16", "norm_out16"), ("norm_v32", "norm_out32")):
        y = D.rmsnorm(golden[src][None, :], golden["norm_g"], eps, half=True)[0]
        r = golden[ref].astype(np.float64)
        ulp = np.spacing(np.abs(r).astype(np.float16)).astype(np.float64)
        assert np.all(np.abs(y - r) <= ulp)


def test_rope_append_attention_matches_reference(golden):
    H, KVH, hd = 16, 8, 128
    qkv = golden["attn_qkv32"].astype(np.float64)
    cos, sin = golden["attn_cos"].astype(np.float64), golden["attn_sin"].astype(np.float64)
    q0 = int(golden["attn_q0"])
    q = qkv[:H * hd].reshape(H, hd)
    k = qkv[H * hd:(H + KVH) * hd].reshape(KVH, hd)
    v = qkv[(H + KVH) * hd:].reshape(KVH, hd)
    qscale = float(golden["attn_qscale"])
    q16 = D.f16(D.rope(q, cos, sin) * qscale)
    k16 = D.f16(D.rope(k, cos, sin))
    v16 = D.f16(v)
    # the appended cache row: fp16 of the rotated k / raw v (the reference rounds each RoPE product in fp32)
    ulp_k = np.spacing(np.abs(golden["attn_knew"]).astype(np.float16)).astype(np.float64)
    assert np.all(np.abs(k16 - golden["attn_knew"].astype(np.float64)) <= ulp_k)
    assert np.array_equal(v16, golden["attn_vnew"].astype(np.float64))
    K = golden["attn_K"].astype(np.float64)
    V = golden["attn_V"].astype(np.float64)
    K[:, q0] = golden["attn_knew"]
    V[:, q0] = golden["attn_vnew"]
    out = D.attention_step(D.f16(q16), K, V, q0 + 1, KVH)
    ref = golden["attn_out"].astype(np.float64)
    # the reference's exp2_soft / fp32 merge and fp16 output: within 2 fp16 ulps plus the q16 rounding effect
    ulp = np.spacing(np.abs(ref).astype(np.float16)).astype(np.float64)
    assert np.all(np.abs(out - ref) <= 2 * ulp + 2e-3 * np.abs(ref).max())


def test_silu_close(golden):
    x = golden["silu_x"].astype(np.float64)
    ref = golden["silu_y"].astype(np.float64)
    assert np.all(np.abs(D.silu(x) - ref) <= 4 * np.finfo(np.float32).eps * (np.abs(ref) + 1e-30))


def test_argmax_first_max(golden):
    assert D.first_argmax(golden["argmax_logits"]) == int(golden["argmax_index"]) == 123


def test_layer_step_matches_reference_fp64_ideal(golden):
    """The oracle's whole layer against the reference's own FP64 decoder-layer step (g17decodestep.ideal)."""
    g = {k[len("layer_in_"):]: golden[k] for k in golden.files if k.startswith("layer_in_")}
    d = g["x"].size
    H, hd = g["k_cache"].shape[0], g["k_cache"].shape[2]
    w = dict(qkv=g["wqkv"].T.astype(np.float64), wo=g["wo"].T.astype(np.float64),
             gate=g["wgate"].T.astype(np.float64), up=g["wup"].T.astype(np.float64),
             down=g["wdown"].T.astype(np.float64))
    pos = int(golden["layer_kv_len"])
    r = D.layer_step64(w, g["x"], g["g1"], g["g2"], g["k_cache"], g["v_cache"], pos,
                       g["rope_cos"].astype(np.float64), g["rope_sin"].astype(np.float64),
                       float(golden["layer_eps"]), H, H)
    for k in ("h1", "qkv32", "k_new", "v_new", "attn", "h", "h2", "act", "out32"):
        ref = golden["layer_out_" + k].astype(np.float64).reshape(r[k].shape)
        # the reference's tables are fp32 cos/sin and the same FP64 algebra: agreement to ~1e-6 relative
        assert np.allclose(r[k], ref, rtol=2e-6, atol=2e-6 * np.abs(ref).max()), k
