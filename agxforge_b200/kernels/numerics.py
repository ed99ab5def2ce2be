"""Shared decode constants (the reference's agxforge/kernels/numerics.py:340-363 rounding points).

    LOG2E, q_scale(head_dim)    the softmax runs in base 2 on q pre-scaled by log2(e)/sqrt(head_dim) (numerics.py:349-351)
    rope_tables(cap, hd, theta) cos/sin [cap, hd/2]: angle p * theta^(-2i/hd) in float64, rounded once to fp32
                                (agxforge/inference/assemble.py:665-668); the library builds the same tables itself
"""
from __future__ import annotations

import math

import numpy as np

LOG2E = 1.4426950408889634


def q_scale(head_dim):
    return np.float32(LOG2E / math.sqrt(head_dim))


def rope_tables(cap, head_dim, theta):
    inv = theta ** (-np.arange(0, head_dim, 2, dtype=np.float64) / head_dim)
    ang = np.arange(cap, dtype=np.float64)[:, None] * inv[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
