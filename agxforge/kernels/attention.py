"""Decode attention for one query row per head (the reference's agxforge/kernels/attention.py: split 86-165, merge
1326-1371, attn_reference 1458-1580), on the B200: split-KV over chunks of the live keys 0..q0 with an online base-2
softmax per chunk and a log-sum-exp merge of the chunks.

    attention(q16, K, V, q0, splits=0)

q16 fp16 [nb, H, hd] already scaled by log2(e)/sqrt(hd) (numerics.q_scale; the softmax is base 2, attention.py:24-25);
K and V fp16 [nb, KVH, cap, hd]; q0 int [nb] (the new token's position; keys 0..q0 are read, q0 clamped to cap - 1,
attention.py:35). GQA: q head h reads KV head h // (H / KVH). Returns fp16 [nb, H * hd].

The reference's names, run on the B200 (numpy in, numpy out, like theirs):

    attn_layout / attn_rope_layout(heads, kv_heads, head_dim, cap, slices)    the layout records (attention.py:53-65,
                                                    168-178); `slices` is kept, the B200 kernel plans its own split
    attn_reference(lay, q16, K, V, q0)              the attention output fp16 [heads, head_dim] (attention.py:1458)
    attn_rope_reference(lay, qkv32, cos, sin, Kc, Vc, q0)
                                                    RoPE, q scale and the K/V append on one fp32 qkv row, then the
                                                    attention: (out, K, V) with the new row in the caches
                                                    (attention.py:1309-1323)
"""
from __future__ import annotations

import ctypes as C

import math

import numpy as np

from agxforge_b200 import _native as N
from agxforge.kernels import qmv as _qmv

LOG2E = 1.4426950408889634


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


def attn_layout(heads=16, kv_heads=8, head_dim=128, cap=272, slices=16):
    """The attention layout record (attention.py:53-65). The B200 kernel takes head_dim 64 or 128 and up to 8 query
    heads per KV head."""
    if head_dim not in (64, 128):
        raise ValueError("attention: head_dim 64 or 128")
    if heads % kv_heads or heads // kv_heads > 8:
        raise ValueError("attention: heads a multiple of kv_heads, at most 8 per KV head")
    if cap < 1:
        raise ValueError("attention: cap >= 1")
    return dict(op="attn", heads=heads, kv_heads=kv_heads, head_dim=head_dim, cap=cap, slices=slices)


def attn_rope_layout(heads=16, kv_heads=8, head_dim=128, cap=272, slices=16):
    """The fused RoPE + append + attention layout record (attention.py:168-178)."""
    return dict(attn_layout(heads, kv_heads, head_dim, cap, slices), rope=True)


def q_scale(head_dim):
    """The base-2 softmax's q scale log2(e)/sqrt(head_dim), rounded to fp32 (numerics.py:349-351)."""
    return np.float32(LOG2E / math.sqrt(head_dim))


def attn_reference(lay, q16, K, V, q0, partials=False, _scalar=False):
    """out fp16 [heads, head_dim]: the attention of q16 (pre-scaled) over keys 0..q0 of K / V [kv_heads, >=q0+1,
    head_dim] (attention.py:1458-1580), by the B200 kernel. `partials` (the reference's per-slice partials) has no
    counterpart: the B200 kernel merges its chunks on chip."""
    import torch
    if partials:
        raise ValueError("attn_reference: the B200 kernel merges its chunks on chip (no slice partials)")
    H, KVH, hd = lay["heads"], lay["kv_heads"], lay["head_dim"]
    Kt = torch.as_tensor(np.asarray(K, np.float16)).cuda()
    Vt = torch.as_tensor(np.asarray(V, np.float16)).cuda()
    q = torch.as_tensor(np.asarray(q16, np.float16).reshape(H, hd)).cuda()
    out = attention(q, Kt, Vt, [min(int(q0), Kt.shape[1] - 1)])
    torch.cuda.synchronize()
    return out.cpu().numpy().reshape(H, hd)


def attn_rope_reference(lay, qkv32, cos, sin, Kc, Vc, q0, partials=False):
    """RoPE + q scale + append of one fp32 qkv row, then the attention (attention.py:1309-1323), on the B200:
    returns (out fp16 [heads, head_dim], K, V) with the new row written at q0 (clamped to cap - 1)."""
    import torch
    if partials:
        raise ValueError("attn_rope_reference: the B200 kernel merges its chunks on chip (no slice partials)")
    H, KVH, hd = lay["heads"], lay["kv_heads"], lay["head_dim"]
    Kt = torch.as_tensor(np.asarray(Kc, np.float16)).cuda().contiguous()
    Vt = torch.as_tensor(np.asarray(Vc, np.float16)).cuda().contiguous()
    cap = Kt.shape[1]
    if Kt.shape != (KVH, cap, hd) or Vt.shape != Kt.shape:
        raise ValueError("attn_rope_reference: Kc and Vc are [kv_heads, cap, head_dim]")
    pos = min(int(q0), cap - 1)
    qkv = torch.as_tensor(np.asarray(qkv32, np.float32).reshape(-1)).cuda()
    if qkv.numel() != (H + 2 * KVH) * hd:
        raise ValueError("attn_rope_reference: qkv32 holds (heads + 2 kv_heads) x head_dim values")
    c = torch.as_tensor(np.asarray(cos, np.float32).reshape(-1)).cuda()
    s = torch.as_tensor(np.asarray(sin, np.float32).reshape(-1)).cuda()
    q16 = torch.empty((H, hd), dtype=torch.float16, device="cuda")
    st = _qmv._stream(torch)
    N.check(N.lib().agxc_rope_append_dev(N.context(0), N.ptr(qkv), H, KVH, hd, cap, pos, N.ptr(c), N.ptr(s),
                                         float(q_scale(hd)), N.ptr(q16), N.ptr(Kt), N.ptr(Vt), st), "rope_append")
    out = attention(q16, Kt, Vt, [pos])
    torch.cuda.synchronize()
    return out.cpu().numpy().reshape(H, hd), Kt.cpu().numpy(), Vt.cpu().numpy()
