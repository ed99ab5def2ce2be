"""Which kernel form each role of the decode step runs (the reference's agxforge/inference/catalog.py:70-233, where a
model config names a per-role variant). On the B200 every role has one form; what varies is the launch plan the
library derives from the shape (K chunks, units per CTA, pipeline stages), reported here for inspection.

    ROLES           the step's kernels in order, with the reference dispatch each one replaces
    launch_plan     the plan of one role: {"kernel", "rows", "k", "epilogue", "prologue"}
"""
from __future__ import annotations

ROLES = [
    ("qkv", "RMSNorm + qkv GEMV + bias + RoPE + KV append", "norm.build_rmsnorm_wide + qmv.build_qmv2 (qkv) + RoPE/append of attention.build_attn_split_rope"),
    ("attn", "split-KV attention + log-sum-exp merge", "attention.build_attn_split_rope (split, merge)"),
    ("wo", "o_proj GEMV + residual (add16)", "qmv.build_qmv2 with_residual('add16')"),
    ("ffn", "RMSNorm + gate/up GEMV + SiLU*mul", "norm.build_rmsnorm_wide + qmv.build_qmv2 (qmv_swiglu_layout)"),
    ("down", "down GEMV + residual (add32_to16)", "qmv.build_qmv2 with_residual('add32_to16')"),
    ("head", "final RMSNorm + vocabulary GEMV + argmax + generation step", "norm + qmv (lm_head) + argmax.build_pass1 + argmax.build_gen"),
]


def launch_plan(shape, role):
    """Rows, K, epilogue and prologue of a role for a models.Model shape."""
    S = shape
    table = {
        "qkv": dict(rows=S.QKV, k=S.D_MODEL, epilogue="bias+rope+append", prologue="rmsnorm(x16)"),
        "wo": dict(rows=S.D_MODEL, k=S.HEADS * S.HEAD_DIM, epilogue="add16", prologue=None),
        "ffn": dict(rows=2 * S.FFN, k=S.D_MODEL, epilogue="swiglu", prologue="rmsnorm(h)"),
        "down": dict(rows=S.D_MODEL, k=S.FFN, epilogue="add32_to16", prologue=None),
        "head": dict(rows=S.VOCAB, k=S.D_MODEL, epilogue="argmax+gen", prologue="rmsnorm(x16)"),
    }
    if role == "attn":
        return dict(kernel="attention", heads=S.HEADS, kv_heads=S.KV_HEADS, head_dim=S.HEAD_DIM)
    if role not in table:
        raise ValueError("unknown role %r" % role)
    return dict(kernel="qmv", **table[role])
