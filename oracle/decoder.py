"""The quantized decoder in FP64 and in half-transport FP64 (numpy; oracle / test infrastructure).

Two policies over the same packs (the reference's validation contract, tools/g17inferencereference.py:22-30,143 and
tools/g17decoderframework.py:11-18):

    fp64            float64 arithmetic, no intermediate rounding (tools/g17decodestep.py:459-489 ``ideal``): the
                    yardstick for the logit bound 0.05 + 0.003*|ref| (tools/g17generationcheck.py:39)
    half            float64 arithmetic with fp16 rounding at every point where the GPU stores an fp16 tensor (x
                    between layers, the normed rows, q/k/v after RoPE, the attention output, the SwiGLU product) and
                    the fp32 RoPE tables the GPU reads: the argmax yardstick

The layer follows the reference's dispatch order and rounding points (agxforge/inference/assemble.py:852-931 QSim.run;
tools/g17decodestep.py:213-273): h1 = fp16(rmsnorm(x16, g1)); qkv = W_qkv h1 (+ bias, Qwen2); rotate-half RoPE at the
token's position on q and k (agxforge/kernels/numerics.py:340-346); q16 = fp16(rope(q) * log2(e)/sqrt(hd)) so the
softmax is base 2 (numerics.py:349-351); k16 = fp16(rope(k)), v16 = fp16(v) appended to the cache; attention over keys
0..pos (agxforge/kernels/attention.py:1659-1668 ``attn_float64``) -> fp16; h = x16 + W_o attn (fp32 storage,
qmv.py:112-120 add16); h2 = fp16(rmsnorm(h, g2)); act = fp16(silu(W_gate h2) * W_up h2) (qmv.py:222-226);
x16' = fp16(h + W_down act) (add32_to16). After the last layer: xf = fp16(rmsnorm(x16, g_final)); logits = W_head xf;
token = first argmax (agxforge/kernels/argmax.py:287-288), or the forced token from the log (argmax.py:141-145).

Because the history is teacher-forced, every position of a sequence is known up front, so the oracle runs the whole
sequence as ONE batched causal pass (position p attends to keys 0..p), which is the same value as stepping the decode
loop token by token.
"""
from __future__ import annotations

import dataclasses
import math

import numpy as np

from oracle import pack as P

F64 = np.float64
LOG2E = 1.4426950408889634


def f16(x):
    """Round to fp16 (RNE) and return the value as float64."""
    with np.errstate(over="ignore"):
        return np.asarray(x, F64).astype(np.float16).astype(F64)


@dataclasses.dataclass
class Shape:
    """A decoder's shapes (agxforge/inference/models.py:26-44 Model record)."""
    d_model: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    eps: float = 1e-6
    rope_theta: float = 1e6
    qkv_bias: bool = False
    tied: bool = False
    qk_norm: bool = False

    @property
    def qkv_rows(self):
        return (self.n_heads + 2 * self.n_kv_heads) * self.head_dim


@dataclasses.dataclass
class Pack:
    """One quantized matrix in the reference format (qmv.py:17-18)."""
    packed: np.ndarray
    s16: np.ndarray
    b16: np.ndarray
    bits: int
    scale_dtype: str
    N: int
    K: int

    def fields(self):
        return P.unpack(self.packed, self.bits, self.N, self.K)

    def w64(self):
        return P.dequant64(self.fields(), self.s16, self.b16, self.scale_dtype)


def rope_tables(cap, head_dim, theta, dtype=np.float32):
    """cos/sin [cap, head_dim/2]: angle p*theta^(-2i/hd) in float64, then rounded to fp32 once
    (agxforge/inference/assemble.py:665-668)."""
    inv = theta ** (-np.arange(0, head_dim, 2, dtype=F64) / head_dim)
    ang = np.arange(cap, dtype=F64)[:, None] * inv[None, :]
    return np.cos(ang).astype(dtype), np.sin(ang).astype(dtype)


def rmsnorm(v, g, eps, half):
    """y = v * rsqrt(mean(v^2) + eps) * g per row (tools/g17decodestep.py:213-234), fp16-rounded under ``half``."""
    v = np.asarray(v, F64)
    r = 1.0 / np.sqrt(np.mean(v * v, axis=-1, keepdims=True) + eps)
    y = v * r * np.asarray(g, F64)
    return f16(y) if half else y


def rope(t, cos, sin):
    """Rotate-half RoPE on the last axis: pairs (i, i + hd/2) (agxforge/kernels/numerics.py:340-346)."""
    h = t.shape[-1] // 2
    x1, x2 = t[..., :h], t[..., h:]
    return np.concatenate([x1 * cos - x2 * sin, x2 * cos + x1 * sin], axis=-1)


def head_norm(t, g, eps):
    """QK-norm (Qwen3): RMSNorm of every head's row over head_dim with a gain shared by the heads, before RoPE and
    without a storage rounding (agxforge/kernels/attention.py:256-265 with_qknorm; tools/g17qwen3.py:216-231)."""
    t = np.asarray(t, F64)
    r = 1.0 / np.sqrt(np.mean(t * t, axis=-1, keepdims=True) + eps)
    return t * r * np.asarray(g, np.float16).astype(F64)


def silu(x):
    return x / (1.0 + np.exp(-x))


def swiglu64(g, u):
    """silu(g) * u over row blocks on the thread pool (float64 throughout)."""
    out = np.empty_like(g)

    def block(r0, r1):
        gg = g[r0:r1]
        out[r0:r1] = gg / (1.0 + np.exp(-gg)) * u[r0:r1]
    P.parallel_rows(g.shape[0], block)
    return out


def attention_causal(q16, k16, v16, n_kv_heads):
    """Base-2 softmax attention of every position over keys 0..p. q16 [T, H, hd] (already scaled by log2e/sqrt(hd)),
    k16/v16 [T, KVH, hd]. Returns [T, H, hd] float64 (attention.py:1659-1668 on every position)."""
    T, H, hd = q16.shape
    G = H // n_kv_heads
    out = np.empty((T, H, hd), F64)
    for h in range(H):
        kv = h // G
        s = q16[:, h, :] @ k16[:, kv, :].T                         # [T, T]
        pr = np.empty_like(s)

        def block(r0, r1):   # rows r0 .. r1-1 see keys 0 .. r (causal)
            sb = s[r0:r1]
            sb[np.arange(r1 - r0)[:, None] + r0 < np.arange(T)[None, :]] = -np.inf
            pr[r0:r1] = np.exp2(sb - sb.max(axis=1, keepdims=True))
        P.parallel_rows(T, block)
        out[:, h, :] = (pr @ v16[:, kv, :]) / pr.sum(axis=1, keepdims=True)
    return out


def attention_step(q16, K, V, nk, n_kv_heads):
    """One query row per head over keys 0..nk-1 (base 2). q16 [H, hd]; K/V [KVH, >=nk, hd]. float64 [H, hd]."""
    H, hd = q16.shape
    G = H // n_kv_heads
    out = np.empty((H, hd), F64)
    for h in range(H):
        kv = h // G
        s = np.asarray(K[kv, :nk], F64) @ np.asarray(q16[h], F64)
        p = np.exp2(s - s.max())
        out[h] = (p @ np.asarray(V[kv, :nk], F64)) / p.sum()
    return out


def layer_step64(w, x, g1, g2, kcache, vcache, pos, cos, sin, eps, n_heads, n_kv_heads, bias=None):
    """One decoder layer for one token at position `pos` over an existing cache (keys 0..pos-1), float64, no
    intermediate rounding (tools/g17decodestep.py:459-489 ``ideal``, generalised to GQA and a qkv bias). Weights are
    [out, in]: w["qkv"], w["wo"], w["gate"], w["up"], w["down"]. Returns the intermediates."""
    x = np.asarray(x, F64)
    hd = kcache.shape[-1]
    H, KVH = n_heads, n_kv_heads
    h1 = rmsnorm(x, g1, eps, False)
    qkv = w["qkv"] @ h1
    if bias is not None:
        qkv = qkv + np.asarray(bias, F64)
    q = qkv[:H * hd].reshape(H, hd)
    k = qkv[H * hd:(H + KVH) * hd].reshape(KVH, hd)
    v = qkv[(H + KVH) * hd:].reshape(KVH, hd)
    qr, kr = rope(q, cos, sin), rope(k, cos, sin)
    K = np.concatenate([np.asarray(kcache, F64)[:, :pos], kr[:, None]], axis=1)
    V = np.concatenate([np.asarray(vcache, F64)[:, :pos], v[:, None]], axis=1)
    attn = attention_step(qr * (LOG2E / math.sqrt(hd)), K, V, pos + 1, KVH).reshape(-1)
    h = x + w["wo"] @ attn
    h2 = rmsnorm(h, g2, eps, False)
    gate, up = w["gate"] @ h2, w["up"] @ h2
    act = silu(gate) * up
    out = h + w["down"] @ act
    return dict(h1=h1, qkv32=qkv, k_new=kr, v_new=v, attn=attn, h=h, h2=h2, act=act, out32=out)


class Model:
    """Weights in the reference's formats: packs per layer (qkv, wo, gate, up, down) and the head; fp16 vectors for
    the embedding table [V, d], the norm gains and (Qwen2) the qkv bias."""

    def __init__(self, shape: Shape, layers, head: Pack, embed, final_gain):
        self.shape = shape
        self.layers = layers          # list of dicts: qkv, wo, gate, up, down (Pack); g1, g2 (fp16); bias (fp16|None)
        self.head = head
        self.embed = np.asarray(embed, np.float16)
        self.final_gain = np.asarray(final_gain, np.float16)

    def forward(self, tokens, policy="fp64", logit_positions=None, keep=False):
        """Teacher-forced causal pass over ``tokens``; returns logits [len(logit_positions), V] (float64) for the
        positions asked (default: all). ``policy`` is "fp64" or "half". With keep=True also returns the per-layer
        K/V (fp16 values under "half") for cache checks."""
        S = self.shape
        half = policy == "half"
        if policy not in ("fp64", "half"):
            raise ValueError("policy is fp64 or half")
        tokens = np.asarray(tokens, np.int64)
        T = tokens.size
        H, KVH, hd = S.n_heads, S.n_kv_heads, S.head_dim
        pos = np.arange(T)
        if half:
            cos, sin = (a.astype(F64) for a in rope_tables(T, hd, S.rope_theta))
        else:
            inv = S.rope_theta ** (-np.arange(0, hd, 2, dtype=F64) / hd)
            ang = pos[:, None].astype(F64) * inv[None, :]
            cos, sin = np.cos(ang), np.sin(ang)
        x = self.embed[tokens].astype(F64)                      # [T, d], fp16 values
        kept = []
        qscale = LOG2E / math.sqrt(hd)
        for L in self.layers:
            h1 = rmsnorm(x, L["g1"].astype(F64), S.eps, half)
            qkv = h1 @ L["qkv"].w64().T
            if L.get("bias") is not None:
                qkv = qkv + np.asarray(L["bias"], np.float16).astype(F64)
            q = qkv[:, :H * hd].reshape(T, H, hd)
            k = qkv[:, H * hd:(H + KVH) * hd].reshape(T, KVH, hd)
            v = qkv[:, (H + KVH) * hd:].reshape(T, KVH, hd)
            if S.qk_norm:
                q, k = head_norm(q, L["qn"], S.eps), head_norm(k, L["kn"], S.eps)
            qr = rope(q, cos[:, None, :], sin[:, None, :]) * qscale
            kr = rope(k, cos[:, None, :], sin[:, None, :])
            if half:
                qr, kr, v = f16(qr), f16(kr), f16(v)
            if keep:
                kept.append((kr.copy(), v.copy()))
            a = attention_causal(qr, kr, v, KVH).reshape(T, H * hd)
            if half:
                a = f16(a)
            h = x + a @ L["wo"].w64().T
            h2 = rmsnorm(h, L["g2"].astype(F64), S.eps, half)
            act = swiglu64(h2 @ L["gate"].w64().T, h2 @ L["up"].w64().T)
            if half:
                act = f16(act)
            x = h + act @ L["down"].w64().T
            if half:
                x = f16(x)
        sel = pos if logit_positions is None else np.asarray(logit_positions, np.int64)
        xf = rmsnorm(x[sel], self.final_gain.astype(F64), S.eps, half)
        logits = xf @ self.head.w64().T
        return (logits, kept) if keep else logits

    def forward_both(self, tokens, logit_positions):
        """Both policies in one pass over the layers (each pack dequantised once): returns (logits FP64, logits
        half-transport, the half-transport final normed rows xf [positions, d] and the head's FP64 weights), for the
        argmax's rounding bound (argmax_rounding_bound)."""
        S = self.shape
        tokens = np.asarray(tokens, np.int64)
        T = tokens.size
        H, KVH, hd = S.n_heads, S.n_kv_heads, S.head_dim
        pos = np.arange(T)
        cos_h, sin_h = (a.astype(F64) for a in rope_tables(T, hd, S.rope_theta))
        inv = S.rope_theta ** (-np.arange(0, hd, 2, dtype=F64) / hd)
        ang = pos[:, None].astype(F64) * inv[None, :]
        cos_f, sin_f = np.cos(ang), np.sin(ang)
        qscale = LOG2E / math.sqrt(hd)
        x = {False: self.embed[tokens].astype(F64), True: self.embed[tokens].astype(F64)}
        for L in self.layers:
            w = {r: L[r].w64() for r in ("qkv", "wo", "gate", "up", "down")}
            for half in (False, True):
                cos, sin = (cos_h, sin_h) if half else (cos_f, sin_f)
                xx = x[half]
                h1 = rmsnorm(xx, L["g1"].astype(F64), S.eps, half)
                qkv = h1 @ w["qkv"].T
                if L.get("bias") is not None:
                    qkv = qkv + np.asarray(L["bias"], np.float16).astype(F64)
                q = qkv[:, :H * hd].reshape(T, H, hd)
                k = qkv[:, H * hd:(H + KVH) * hd].reshape(T, KVH, hd)
                v = qkv[:, (H + KVH) * hd:].reshape(T, KVH, hd)
                if S.qk_norm:
                    q, k = head_norm(q, L["qn"], S.eps), head_norm(k, L["kn"], S.eps)
                qr = rope(q, cos[:, None, :], sin[:, None, :]) * qscale
                kr = rope(k, cos[:, None, :], sin[:, None, :])
                if half:
                    qr, kr, v = f16(qr), f16(kr), f16(v)
                a = attention_causal(qr, kr, v, KVH).reshape(T, H * hd)
                if half:
                    a = f16(a)
                h = xx + a @ w["wo"].T
                h2 = rmsnorm(h, L["g2"].astype(F64), S.eps, half)
                act = swiglu64(h2 @ w["gate"].T, h2 @ w["up"].T)
                if half:
                    act = f16(act)
                xn = h + act @ w["down"].T
                x[half] = f16(xn) if half else xn
            del w
        sel = np.asarray(logit_positions, np.int64)
        W = self.head.w64()
        xf64 = rmsnorm(x[False][sel], self.final_gain.astype(F64), S.eps, False)
        xfh = rmsnorm(x[True][sel], self.final_gain.astype(F64), S.eps, True)
        return xf64 @ W.T, xfh @ W.T, xfh, W


def first_argmax(v):
    """The first index of the maximum (np.argmax's rule; agxforge/kernels/argmax.py:287-288)."""
    return int(np.argmax(np.asarray(v)))


def top2_margin(v):
    """max - second max of a logit row (how close the greedy choice is to a tie)."""
    v = np.asarray(v, F64)
    i = int(np.argmax(v))
    w = np.delete(v, i)
    return float(v[i] - w.max())


def argmax_rounding_bound(W, xfh, i, j, K=None):
    """How far apart two logits i and j of one step may be and still swap order between the GPU and the
    half-transport oracle through rounding alone. The two sides store the same fp16 points; after the last layer the
    final normed row xf is fp16 on both, and a pre-rounding value that lands on the other side of an fp16 rounding
    boundary moves an element by one fp16 ulp. Assuming at most that (one ulp16 per element of xf) plus the fp32
    accumulation of the K-term dot products (K eps32 relative, the textbook gamma_K bound), each logit moves by at
    most
        d_r = sum_k |W_rk| ulp16(xf_k) + K eps32 sum_k |W_rk xf_k|,
    and the order of i and j can only flip if their margin is at most d_i + d_j."""
    xfh = np.asarray(xfh, F64)
    ulp = np.spacing(np.abs(xfh).astype(np.float16)).astype(F64)
    K = xfh.size if K is None else K
    eps32 = float(np.finfo(np.float32).eps)

    def d(r):
        wr = np.abs(np.asarray(W[r], F64))
        return float(wr @ ulp + K * eps32 * (wr @ np.abs(xfh)))
    return d(i) + d(j)


def logit_bound(ref):
    """The reference's logit budget: |err| <= 0.05 + 0.003*|ref| (tools/g17generationcheck.py:39)."""
    return 0.05 + 0.003 * np.abs(np.asarray(ref, F64))
