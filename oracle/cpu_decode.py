"""The reference's CPU decode step as a numpy FP32 port — the timed CPU baseline (oracle / test infrastructure).

The reference's own CPU implementation of this path is its simulator QSim, which runs every dispatch of the decode
graph through that kernel's numpy reference (agxforge/inference/assemble.py:852-931): rmsnorm_wide_reference ->
qmv2_ksplit_reference (qkv) -> attn_rope_reference -> qmv2_ksplit_reference + residual_reference (add16) -> norm ->
qmv_swiglu_reference -> qmv2_ksplit_reference + residual_reference (add32_to16) -> final norm -> head -> np.argmax.
Those references are not importable where the baseline runs, so this module restates the same chain in plain numpy
FP32: each projection dequantises its pack row-block by row-block (w = q*s + b, agxforge/kernels/qmv.py:1699-1750)
and forms the fp32 dot products, with the reference's storage rounding points (fp16 x, normed rows, q/k/v, attention
output, SwiGLU product). Row blocks run on a thread pool over the host's cores, as the reference's references do
(qmv.py:1641-1648, G17_REF_THREADS).

    host_packs(shape, bits, scale_dtype, seed)   the model's packs made on the host: seeded N(0, 0.02) fp32 weights
                                                 quantised by oracle.pack (the reference's quantize), fp16 embedding,
                                                 unit gains; no device and no native library involved
    CpuDecoder.decode_token(x16, pos)            one whole decode step (every layer, the head, the first argmax)
"""
from __future__ import annotations

import math
import os
import time
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from oracle import pack as P

F32 = np.float32


ROLE_SEED = {"qkv": 0, "wo": 1, "gate": 2, "up": 3, "down": 4, "head": 5}


def host_packs(shape, bits, scale_dtype, seed, threads=None, std=0.02):
    """Every pack, gain and the embedding of a synthetic model, generated and quantised on the host (matrices in
    parallel over the cores; numpy's generators and array kernels release the GIL). Keys as DecodeModel.packs."""
    S = shape
    jobs = [((l, role), n, k) for l in range(S.LAYERS) for role, n, k in S.matrices()]
    jobs.append(((None, "head"), S.VOCAB, S.D_MODEL))
    out = {}

    def make(job):
        (l, role), n, k = job
        rng = np.random.default_rng([seed, 1000 if l is None else l, ROLE_SEED[role]])
        W = rng.standard_normal((n, k), dtype=F32) * F32(std)
        a, sc, b, _ = P.quantize(W, bits, scale_dtype=scale_dtype)
        return job[0], (a, sc, b)
    with ThreadPoolExecutor(threads or os.cpu_count() or 1) as pool:
        for key, val in pool.map(make, jobs):
            out[key] = val
    rng = np.random.default_rng([seed, 99])
    out["embed"] = (rng.standard_normal((S.VOCAB, S.D_MODEL), dtype=F32) * F32(std)).astype(np.float16)
    for l in range(S.LAYERS):
        out[(l, "attn_gain")] = np.ones(S.D_MODEL, np.float16)
        out[(l, "ffn_gain")] = np.ones(S.D_MODEL, np.float16)
        if S.QKV_BIAS:
            out[(l, "qkv_bias")] = (rng.standard_normal(S.QKV, dtype=F32) * F32(std)).astype(np.float16)
    out["final_gain"] = np.ones(S.D_MODEL, np.float16)
    return out


class CpuDecoder:
    def __init__(self, shape, packs, bits, scale_dtype, cap, threads=None):
        self.S = shape
        self.k = packs
        self.bits = bits
        self.sdt = scale_dtype
        self.cap = cap
        self.threads = threads or os.cpu_count() or 1
        self.pool = ThreadPoolExecutor(self.threads)
        S = shape
        self.K = np.zeros((S.LAYERS, S.KV_HEADS, cap, S.HEAD_DIM), np.float16)
        self.V = np.zeros_like(self.K)
        inv = S.ROPE_THETA ** (-np.arange(0, S.HEAD_DIM, 2, dtype=np.float64) / S.HEAD_DIM)
        ang = np.arange(cap, dtype=np.float64)[:, None] * inv[None, :]
        self.cos, self.sin = np.cos(ang).astype(F32), np.sin(ang).astype(F32)

    def matvec(self, key, n, kk, x):
        """y = W x in fp32 for one pack, dequantised in row blocks on the thread pool."""
        packed, s16, b16 = self.k[key]
        per = 32 // self.bits
        x = np.asarray(x, F32)
        y = np.empty(n, F32)
        rows = max(16, (1 << 18) // max(kk, 1))

        def block(r0):
            r1 = min(n, r0 + rows)
            q = P.unpack(packed[r0:r1], self.bits, r1 - r0, kk).astype(F32)
            s = P.from_16(s16[r0:r1], self.sdt)
            b = P.from_16(b16[r0:r1], self.sdt)
            w = (q.reshape(r1 - r0, kk // 64, 64) * s[..., None] + b[..., None]).reshape(r1 - r0, kk)
            y[r0:r1] = w @ x
        list(self.pool.map(block, range(0, n, rows)))
        return y

    @staticmethod
    def rmsnorm(v, g, eps):
        v = np.asarray(v, F32)
        r = F32(1.0) / np.sqrt(np.mean(v * v, dtype=F32) + F32(eps))
        return ((v * r) * np.asarray(g, F32)).astype(np.float16).astype(F32)

    def layer(self, l, x16, pos):
        S, k = self.S, self.k
        H, KVH, hd, d = S.HEADS, S.KV_HEADS, S.HEAD_DIM, S.D_MODEL
        h1 = self.rmsnorm(x16, k[(l, "attn_gain")], S.EPS)
        qkv = self.matvec((l, "qkv"), S.QKV, d, h1)
        if (l, "qkv_bias") in k:
            qkv = qkv + k[(l, "qkv_bias")].astype(F32)
        c, s = self.cos[pos], self.sin[pos]

        def rot(t):
            a, b = t[..., :hd // 2], t[..., hd // 2:]
            return np.concatenate([a * c - b * s, b * c + a * s], axis=-1)
        q = qkv[:H * hd].reshape(H, hd)
        kk = qkv[H * hd:(H + KVH) * hd].reshape(KVH, hd)
        vv = qkv[(H + KVH) * hd:].reshape(KVH, hd)
        q16 = (rot(q) * F32(1.4426950408889634 / math.sqrt(hd))).astype(np.float16).astype(F32)
        self.K[l, :, pos] = rot(kk).astype(np.float16)
        self.V[l, :, pos] = vv.astype(np.float16)
        G = H // KVH
        out = np.empty((H, hd), F32)
        for h in range(H):
            Kh = self.K[l, h // G, :pos + 1].astype(F32)
            sc = Kh @ q16[h]
            p = np.exp2(sc - sc.max())
            out[h] = (p @ self.V[l, h // G, :pos + 1].astype(F32)) / p.sum()
        attn = out.reshape(-1).astype(np.float16).astype(F32)
        h = self.matvec((l, "wo"), d, H * hd, attn) + x16
        h2 = self.rmsnorm(h, k[(l, "ffn_gain")], S.EPS)
        g = self.matvec((l, "gate"), S.FFN, d, h2)
        u = self.matvec((l, "up"), S.FFN, d, h2)
        act = (g / (F32(1) + np.exp(-g)) * u).astype(np.float16).astype(F32)
        return (self.matvec((l, "down"), d, S.FFN, act) + h).astype(np.float16).astype(F32)

    def head(self, x16):
        xf = self.rmsnorm(x16, self.k["final_gain"], self.S.EPS)
        return self.matvec((None, "head"), self.S.VOCAB, self.S.D_MODEL, xf)

    def fill_history(self, n, seed=0):
        """KV rows 0 .. n-1 of every layer hold seeded N(0, 1) fp16 values (the bench's device-filled history)."""
        rng = np.random.default_rng(seed)
        self.K[:, :, :n] = rng.standard_normal(self.K[:, :, :n].shape, dtype=F32).astype(np.float16)
        self.V[:, :, :n] = rng.standard_normal(self.V[:, :, :n].shape, dtype=F32).astype(np.float16)

    def decode_token(self, token, pos):
        """One whole decode step of the token at position `pos`: x = embedding(token), every layer (appending its K/V
        row at pos), the final norm, the head and the first argmax. Returns the next token."""
        x = self.k["embed"][int(token)].astype(F32)
        for l in range(self.S.LAYERS):
            x = self.layer(l, x, pos)
        return int(np.argmax(self.head(x)))

    def timed_sample(self, layers, pos, seed=0):
        """Time `layers` layers and the head of one decode step at position `pos` (the KV rows before pos hold
        seeded values). Returns (seconds per layer, seconds for the head)."""
        rng = np.random.default_rng(seed)
        self.K[:, :, :pos] = rng.standard_normal(self.K[:, :, :pos].shape).astype(np.float16)
        self.V[:, :, :pos] = rng.standard_normal(self.V[:, :, :pos].shape).astype(np.float16)
        x = self.k["embed"][int(rng.integers(0, self.S.VOCAB))].astype(F32)
        t0 = time.perf_counter()
        for l in range(layers):
            x = self.layer(l, x, pos)
        t1 = time.perf_counter()
        lg = self.head(x)
        t2 = time.perf_counter()
        self.last_token = int(np.argmax(lg))
        return (t1 - t0) / layers, t2 - t1
