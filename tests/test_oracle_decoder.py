"""The oracle's teacher-forced causal pass equals stepping the layer token by token (layer_step64, pinned against the
reference's FP64 step), and the CPU-baseline port agrees with the oracle within fp32/fp16 rounding."""
import math

import numpy as np

from oracle import decoder as D
from oracle import pack as P


def tiny_model(seed=0, bits=4, bias=True, L=2):
    rng = np.random.default_rng(seed)
    shape = D.Shape(d_model=128, n_layers=L, n_heads=4, n_kv_heads=2, head_dim=32, ffn=256, vocab=96, eps=1e-6,
                    rope_theta=1e6, qkv_bias=bias)

    def pk(n, k):
        a, s, b, _ = P.quantize((rng.standard_normal((n, k)) * 0.05).astype(np.float32), bits, scale_dtype="fp16")
        return D.Pack(a, s, b, bits, "fp16", n, k)
    layers = []
    for _ in range(L):
        layers.append(dict(qkv=pk(shape.qkv_rows, 128), wo=pk(128, 128), gate=pk(256, 128), up=pk(256, 128),
                           down=pk(128, 256), g1=(1 + 0.1 * rng.standard_normal(128)).astype(np.float16),
                           g2=(1 + 0.1 * rng.standard_normal(128)).astype(np.float16),
                           bias=(rng.standard_normal(shape.qkv_rows) * 0.02).astype(np.float16) if bias else None))
    emb = (rng.standard_normal((96, 128)) * 0.5).astype(np.float16)
    return D.Model(shape, layers, pk(96, 128), emb, (1 + 0.1 * rng.standard_normal(128)).astype(np.float16))


def test_causal_pass_equals_token_steps():
    m = tiny_model()
    S = m.shape
    toks = [3, 17, 40, 5, 90, 11, 64]
    T = len(toks)
    ref = m.forward(toks, "fp64")
    inv = S.rope_theta ** (-np.arange(0, S.head_dim, 2, dtype=np.float64) / S.head_dim)
    caches = [(np.zeros((S.n_kv_heads, T, S.head_dim)), np.zeros((S.n_kv_heads, T, S.head_dim))) for _ in m.layers]
    for p, t in enumerate(toks):
        x = m.embed[t].astype(np.float64)
        cos, sin = np.cos(p * inv), np.sin(p * inv)
        for l, L in enumerate(m.layers):
            w = {r: L[r].w64() for r in ("qkv", "wo", "gate", "up", "down")}
            r = D.layer_step64(w, x, L["g1"], L["g2"], caches[l][0], caches[l][1], p, cos, sin, S.eps, S.n_heads,
                               S.n_kv_heads, bias=L["bias"])
            caches[l][0][:, p] = r["k_new"]
            caches[l][1][:, p] = r["v_new"]
            x = r["out32"]
        lg = m.head.w64() @ D.rmsnorm(x, m.final_gain, S.eps, False)
        assert np.allclose(lg, ref[p], rtol=1e-9, atol=1e-9)


def test_half_policy_close_to_fp64():
    m = tiny_model(1)
    toks = list(range(0, 60, 7))
    a = m.forward(toks, "fp64")
    b = m.forward(toks, "half")
    assert np.all(np.abs(a - b) <= D.logit_bound(a))


def test_cpu_port_matches_oracle():
    from oracle.cpu_decode import CpuDecoder
    from agxforge.inference.models import Model as MShape
    m = tiny_model(2)
    S = m.shape
    shape = MShape("tiny", S.d_model, S.n_layers, S.n_heads, S.n_kv_heads, S.head_dim, S.ffn, S.vocab, S.rope_theta,
                   S.eps, QKV_BIAS=True)
    packs = {"embed": m.embed, "final_gain": m.final_gain, (None, "head"): (m.head.packed, m.head.s16, m.head.b16)}
    for l, L in enumerate(m.layers):
        for r in ("qkv", "wo", "gate", "up", "down"):
            packs[(l, r)] = (L[r].packed, L[r].s16, L[r].b16)
        packs[(l, "attn_gain")], packs[(l, "ffn_gain")], packs[(l, "qkv_bias")] = L["g1"], L["g2"], L["bias"]
    cpu = CpuDecoder(shape, packs, 4, "fp16", 16, threads=2)
    toks = [4, 8, 15, 16, 23, 42]
    ref = m.forward(toks, "fp64")
    for p, t in enumerate(toks):
        x = m.embed[t].astype(np.float32)
        for l in range(S.n_layers):
            x = cpu.layer(l, x, p)
        lg = cpu.head(x)
        assert np.all(np.abs(lg - ref[p]) <= D.logit_bound(ref[p]))
