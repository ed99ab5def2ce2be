"""Generate tests/golden/ref_kernels.npz from the reference's own CPU kernel references.

Usage:  python tests/golden/make_golden.py <path of an AGXForge checkout>

Imports the reference's ``agxforge.kernels`` modules unchanged from the given checkout (they are pure numpy) and
records, on small seeded inputs, the values of the functions that define the quantized decode path:

    qmv.quantize             (agxforge/kernels/qmv.py:1854)  bf16 scale/bias packs, 4 and 8 bits
    qmv._fma32v              (qmv.py:1537)                   the dequantised fp32 weights fma(q, s, b)
    qmv.qmv2_ksplit_reference (qmv.py:1838)                  the split-K GEMV in the reference kernel's fp32 order
    qmv.qmv_swiglu_reference (qmv.py:222)                    the fused gate/up + SiLU*mul
    qmv.residual_reference   (qmv.py:169)                    add16 / add32_to16 epilogues
    norm.rmsnorm_wide_reference (agxforge/kernels/norm.py:185) the wide RMSNorm (fp16 and fp32 input rows)
    attention.attn_rope_reference (agxforge/kernels/attention.py:1309) RoPE + KV append + split softmax + merge
    numerics.silu            (agxforge/kernels/numerics.py:354)
    tools/g17decodestep.ideal (tools/g17decodestep.py:459-489) one whole decoder layer in FP64
    argmax.argmax_reference  (agxforge/kernels/argmax.py:287) including a tie

The checkout is only read. The npz is committed, so the GPU box (which has no checkout) and the CPU tests use it.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
F32 = np.float32


def main(ref_root):
    sys.path.insert(0, ref_root)
    from agxforge.kernels import argmax, attention, norm, numerics, qmv

    out = {}
    rng = np.random.default_rng(20261201)

    # ---- quantize (bf16 scale/bias, MLX affine group 64) + the dequantised fp32 weights
    for bits in (4, 8):
        W = (rng.standard_normal((48, 256)) * 0.02).astype(F32)
        W[3, 0:64] = F32(0.0125)                       # a constant group: scale 1.0, all fields 0
        W[5, 64:128] *= F32(50.0)                      # a wide-range group
        packed, s16, b16, q = qmv.quantize(W, bits=bits)
        s32, b32 = qmv._from_bf16(s16), qmv._from_bf16(b16)
        w_dq = qmv._fma32v(q.astype(np.float64), np.repeat(s32, 64, 1), np.repeat(b32, 64, 1))
        out.update({"quant%d_W" % bits: W, "quant%d_packed" % bits: packed, "quant%d_s16" % bits: s16,
                    "quant%d_b16" % bits: b16, "quant%d_q" % bits: q.astype(np.uint8), "quant%d_wdq" % bits: w_dq})

    # ---- split-K GEMV (the delivered v2 form: coalesced trips, wpt 2, split-K 2), x holding fp16 values
    for bits in (4, 8):
        N, K = 64, 1024
        W = (rng.standard_normal((N, K)) * 0.02).astype(F32)
        packed, s16, b16, q = qmv.quantize(W, bits=bits)
        x = rng.standard_normal(K).astype(np.float16).astype(F32)
        lay = dict(Nout=N, Kq=K, bits=bits, group=64, per_word=32 // bits, wpt=2, coalesced=True, sgs=2, ksplit=True)
        y = qmv.qmv2_ksplit_reference(lay, x, q, s16, b16)
        out.update({"qmv%d_packed" % bits: packed, "qmv%d_s16" % bits: s16, "qmv%d_b16" % bits: b16,
                    "qmv%d_x" % bits: x, "qmv%d_y" % bits: y})

    # ---- fused gate/up + SiLU*mul: 2F rows (gate rows then up rows)
    F, K = 32, 1024
    W = (rng.standard_normal((2 * F, K)) * 0.02).astype(F32)
    packed, s16, b16, q = qmv.quantize(W, bits=4)
    x = rng.standard_normal(K).astype(np.float16).astype(F32)
    lay = dict(Nout=2 * F, Kq=K, bits=4, group=64, per_word=8, wpt=2, coalesced=True, sgs=2, ksplit=True,
               swiglu=True, ffn=F)
    act = qmv.qmv_swiglu_reference(lay, x, q, s16, b16)
    out.update(swiglu_packed=packed, swiglu_s16=s16, swiglu_b16=b16, swiglu_x=x, swiglu_act=np.asarray(act, np.float16))

    # ---- residual epilogues
    y = rng.standard_normal(256).astype(F32)
    x16 = rng.standard_normal(256).astype(np.float16)
    h32 = rng.standard_normal(256).astype(F32)
    out.update(res_y=y, res_x16=x16, res_h32=h32,
               res_add16=qmv.residual_reference(dict(res="add16"), y, x16=x16),
               res_add32_to16=np.asarray(qmv.residual_reference(dict(res="add32_to16"), y, h32=h32), np.float16))

    # ---- wide RMSNorm, fp16 and fp32 input rows
    spec = numerics.LayerSpec()                                    # d 2048, eps 1e-5, fp16 storage
    v16 = rng.standard_normal(2048).astype(np.float16).astype(F32)
    v32 = (rng.standard_normal(2048) * 3.0).astype(F32)
    g = (1.0 + 0.1 * rng.standard_normal(2048)).astype(np.float16).astype(F32)
    out.update(norm_v16=v16, norm_v32=v32, norm_g=g, norm_eps=np.float64(spec.norm_eps),
               norm_out16=np.asarray(norm.rmsnorm_wide_reference(v16, g, spec), np.float16),
               norm_out32=np.asarray(norm.rmsnorm_wide_reference(v32, g, spec), np.float16))

    # ---- RoPE + append + attention (16 q heads / 8 KV heads / hd 128), position q0
    cap, q0 = 64, 40
    lay = attention.attn_rope_layout(heads=16, kv_heads=8, head_dim=128, cap=cap, slices=16)
    qkv32 = (rng.standard_normal(32 * 128) * 2.0).astype(F32)
    inv = 1e6 ** (-np.arange(0, 128, 2, dtype=np.float64) / 128)
    cos = np.cos(q0 * inv).astype(F32)
    sin = np.sin(q0 * inv).astype(F32)
    Kc = rng.standard_normal((8, cap, 128)).astype(np.float16)
    Vc = rng.standard_normal((8, cap, 128)).astype(np.float16)
    Kc[:, q0:] = 0
    Vc[:, q0:] = 0
    attn, K2, V2 = attention.attn_rope_reference(lay, qkv32, cos, sin, Kc.astype(F32), Vc.astype(F32), q0)
    out.update(attn_qkv32=qkv32, attn_cos=cos, attn_sin=sin, attn_K=Kc, attn_V=Vc, attn_q0=np.int64(q0),
               attn_out=np.asarray(attn, np.float16), attn_knew=np.asarray(K2[:, q0], np.float16),
               attn_vnew=np.asarray(V2[:, q0], np.float16),
               attn_qscale=np.float32(numerics.q_scale(numerics.MILESTONE)))

    # ---- SiLU and argmax (first maximum wins a tie)
    sx = (rng.standard_normal(512) * 4.0).astype(F32)
    logits = rng.standard_normal(1000).astype(F32)
    logits[[123, 777]] = F32(9.5)
    out.update(silu_x=sx, silu_y=numerics.silu(sx), argmax_logits=logits,
               argmax_index=np.int64(argmax.argmax_reference(logits)))

    # ---- one whole decoder layer in FP64 (tools/g17decodestep.py:459-489 ``ideal``): MHA, d 256, 2 heads of 128,
    # FFN 512, 5 cached positions (the new token at position 5)
    sys.path.insert(0, os.path.join(ref_root, "tools"))
    import g17decodestep as DS
    spec = numerics.LayerSpec(d_model=256, n_heads=2, head_dim=128, ffn_dim=512, kv_len=5)
    inp = DS.make_inputs(spec, seed=3)
    ide = DS.ideal(spec, inp)
    for k_, v_ in inp.items():
        out["layer_in_" + k_] = np.asarray(v_)
    for k_ in ("h1", "qkv32", "k_new", "v_new", "attn", "h", "h2", "act", "out32"):
        out["layer_out_" + k_] = np.asarray(ide[k_])
    out.update(layer_eps=np.float64(spec.norm_eps), layer_rope_base=np.float64(spec.rope_base),
               layer_kv_len=np.int64(spec.kv_len))

    path = os.path.join(HERE, "ref_kernels.npz")
    np.savez_compressed(path, **out)
    print("wrote %s (%d arrays, %d bytes)" % (path, len(out), os.path.getsize(path)))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit(__doc__)
    main(sys.argv[1])
