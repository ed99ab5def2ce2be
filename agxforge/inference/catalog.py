"""Which kernel form each role of the decode step runs, and its layout (the reference's
agxforge/inference/catalog.py:70-233).

In the reference a model config names a per-role G17 code variant ({"ks": S, "lean": True, ...}) and the catalog turns
(bits, role, variant) into that variant's layout record. On the B200 every role has one kernel form; the launch plan
(K chunks, row tiles per unit, ring stages, CTAs) is chosen by the library's planner from the shape. So:

    qmv_layout(bits, role, variant=None, shape)   (layout, flags) for "qkv", "wo_res1", "ffn", "w2_res2" (the
                                                  reference's role names): the kernels.qmv layout record with the
                                                  role's fused prologue / epilogue; `variant` is recorded, not needed
    head_layout(bits, variant=None, shape)        (layout, variant) of the vocabulary head (final norm + GEMV + argmax)
    norm_layout(in_dtype, out32, seed, shape)     the RMSNorm record (fused into the GEMV that consumes it)
    attn_layout(cap, flags="", shape)             the attention record (RoPE + append + split-KV attention)
    plan(model)                                   the launch plan the library chose for each role of a built
                                                  DecodeModel (its planner's output, DecodeModel.plan_info())

`shape` defaults to the InternLM2.5-1.8B record, the model the reference's catalog is written for (catalog.py:33-42).
"""
from __future__ import annotations

from agxforge.inference import models
from agxforge.kernels import attention, qmv

ROLES = ("qkv", "wo_res1", "ffn", "w2_res2")


def qmv_layout(bits, role, variant=None, shape=models.INTERNLM25_18B):
    S = shape
    variant = dict(variant or {})
    if role == "qkv":
        lay = qmv.with_norm(qmv.qmv_layout(S.QKV, S.D_MODEL, bits, rows=16), "half")
        lay.update(epilogue="bias+rope+append" if S.QKV_BIAS else "rope+append")
    elif role == "wo_res1":
        lay = qmv.with_residual(qmv.qmv_layout(S.D_MODEL, S.HEADS * S.HEAD_DIM, bits, rows=16), "add16")
    elif role == "ffn":
        lay = qmv.with_norm(qmv.qmv_swiglu_layout(S.FFN, S.D_MODEL, bits, rows=16), "float")
    elif role == "w2_res2":
        lay = qmv.with_residual(qmv.qmv_layout(S.D_MODEL, S.FFN, bits, rows=16), "add32_to16")
    else:
        raise ValueError("unknown projection role %r" % role)
    lay["eps"] = S.EPS
    lay["variant"] = variant
    return lay, sorted(k for k, v in variant.items() if v)


def head_layout(bits, variant=None, shape=models.INTERNLM25_18B):
    S = shape
    lay = qmv.with_norm(qmv.qmv_layout(S.VOCAB, S.D_MODEL, bits, rows=16), "half")
    lay.update(eps=S.EPS, epilogue="argmax+gen", tied=S.TIED)
    return lay, dict(variant or {})


def norm_layout(in_dtype, out32, seed, shape=models.INTERNLM25_18B):
    if in_dtype not in ("half", "float"):
        raise ValueError("norm_layout: in_dtype half or float")
    return dict(op="rmsnorm", d=shape.D_MODEL, in_dtype=in_dtype, out32=bool(out32), eps=shape.EPS, seed=bool(seed))


def attn_layout(cap, flags="", shape=models.INTERNLM25_18B):
    lay = attention.attn_rope_layout(shape.HEADS, shape.KV_HEADS, shape.HEAD_DIM, cap)
    lay["flags"] = flags
    return lay


def plan(model):
    """The library's launch plan for each role of a built DecodeModel, keyed by role."""
    return model.plan_info()
