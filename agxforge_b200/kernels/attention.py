"""Decode attention for one query row per head (the reference's agxforge/kernels/attention.py: split 86-165, merge
1326-1371, attn_reference 1458-1580), on the B200: split-KV over chunks of the live keys 0..q0 with an online base-2
softmax per chunk and a log-sum-exp merge of the chunks.

    attention(q16, K, V, q0, splits=0)

q16 fp16 [nb, H, hd] already scaled by log2(e)/sqrt(hd) (numerics.q_scale; the softmax is base 2, attention.py:24-25);
K and V fp16 [nb, KVH, cap, hd]; q0 int [nb] (the new token's position; keys 0..q0 are read, q0 clamped to cap - 1,
attention.py:35). GQA: q head h reads KV head h // (H / KVH). Returns fp16 [nb, H * hd].
"""
from __future__ import annotations

import ctypes as C

from agxforge_b200 import _native as N
from agxforge_b200.kernels import qmv as _qmv


def attention(q16, K, V, q0, splits=0, device=0):
    import torch
    if q16.dim() == 2:
        q16, K, V = q16[None], K[None], V[None]
    nb, H, hd = q16.shape
    _, KVH, cap, hd2 = K.shape
    if hd2 != hd or V.shape != K.shape or K.shape[0] != nb:
        raise ValueError("attention: K and V are [nb, kv_heads, cap, head_dim] matching q")
    if hd not in (64, 128):
        raise ValueError("attention: head_dim 64 or 128")
    if H % KVH or H // KVH > 8:
        raise ValueError("attention: heads a multiple of kv_heads, at most 8 per KV head")
    if q16.dtype != torch.float16 or K.dtype != torch.float16 or V.dtype != torch.float16:
        raise ValueError("attention: fp16 q, K, V")
    q0t = torch.as_tensor(q0, dtype=torch.int32, device=q16.device).reshape(-1).contiguous()
    if q0t.numel() != nb:
        raise ValueError("attention: one q0 per sequence")
    out = torch.empty((nb, H * hd), dtype=torch.float16, device=q16.device)
    q16, K, V = q16.contiguous(), K.contiguous(), V.contiguous()
    N.check(N.lib().agxc_attention_dev(N.context(device), nb, H, KVH, hd, cap, N.ptr(q0t), N.ptr(q16), N.ptr(K),
                                       N.ptr(V), N.ptr(out), int(splits),
                                       _qmv._stream(torch)), "attention")
    return out
