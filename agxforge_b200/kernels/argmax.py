"""Argmax and the device-resident generation step (the reference's agxforge/kernels/argmax.py).

On the B200 the argmax is fused into the vocabulary GEMV (each CTA keeps the first maximum of its rows, the last CTA
to finish reduces the CTAs' pairs) and the generation step runs in that same last CTA: token = the pending forced
token, else the logged prompt token at q0 + 1, else the first maximum; the token is logged at q0 + 1, its embedding
row becomes the next x, and q0 advances, clamped to cap - 1 (argmax.py:133-215; assemble.py:918-930).

    TOKEN_UNSET     a free log entry (0xFFFFFFFF)
    choose(...)     the rule itself, for host-side bookkeeping and documentation
"""
from __future__ import annotations

from agxforge_b200._native import TOKEN_UNSET


def choose(forced, logged, argmax_index):
    """The generation step's token rule (argmax.py:141-145 plus the per-step forced input)."""
    if forced is not None and forced != TOKEN_UNSET:
        return int(forced)
    if logged is not None and logged != TOKEN_UNSET:
        return int(logged)
    return int(argmax_index)


def first_max_wins(a_value, a_index, b_value, b_index):
    """The tie rule of every argmax reduction here: the larger value, and on a tie the smaller index."""
    return (a_value, a_index) if (a_value > b_value or (a_value == b_value and a_index < b_index)) else (b_value, b_index)
