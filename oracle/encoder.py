"""The BERT sentence encoder (MiniLM-L6 shape) in FP64 and half-transport FP64 (numpy; oracle / test
infrastructure only — never imported by the package).

Restates the reference's complete-encoder reference, tools/g17inferencereference.py:18-99 ``graph_reference``, over
the graph that agxforge/g17/inferencegraph.py:208-289 ``import_graph`` builds for a BERT checkpoint with sentence
pooling, generalised from its single 32-token sequence to a batch [B, S] of sequences with 0/1 padding masks:

    embedding   x = word[ids] + position[pos] + token_type[types]; LayerNorm               (inferencegraph.py:224-234)
    per layer   q, k, v = linear(x) (weights [out, in], bias); attention over the keys whose mask is 1, scale
                1/sqrt(head_width), softmax; o = linear(ctx); x = LayerNorm(o + x);
                u = gelu_erf(linear(x)); d = linear(u); x = LayerNorm(d + x)                  (inferencegraph.py:236-279)
    pooling     mean of x over the rows whose mask is 1 (denominator >= 1e-9), then x / max(||x||, 1e-12)
                                                                                             (inferencegraph.py:284-286)

LayerNorm: (x - mean) / sqrt(mean((x - mean)^2) + eps) * g + b (g17inferencereference.py:58-62). Policies
(g17inferencereference.py:22-30): ``fp64`` = float64 throughout ("original_fp64"); ``half`` = float64 with the
operands of every linear (the activation rows and the weights) rounded to fp16 first ("half_transport_fp64") — the
yardstick of the bound 2e-4 * (1 + |ref|) (g17inferencereference.py:155), with cosine >= 0.999 against fp64.

``make_params`` draws a seeded random-init parameter set in the checkpoint's names (HF BertModel), every value
fp16-representable, so the device model (fp16 parameters) and both policies see the same numbers.
"""
from __future__ import annotations

import math

import numpy as np

F64 = np.float64

MINILM_L6 = dict(model_type="bert", architectures=["BertModel"], hidden_size=384, num_attention_heads=12,
                 intermediate_size=1536, num_hidden_layers=6, vocab_size=30522, max_position_embeddings=512,
                 type_vocab_size=2, layer_norm_eps=1e-12, hidden_act="gelu")


def _f16(x):
    return np.asarray(x, F64).astype(np.float16).astype(F64)


def make_params(seed, config=None, std=0.02):
    """Seeded random-init parameters (names as in the checkpoint): linear weights, biases and embeddings
    N(0, std); LayerNorm gains 1 + N(0, std), biases N(0, std). Every value is fp16-representable (float32 arrays)."""
    c = dict(MINILM_L6, **(config or {}))
    rng = np.random.default_rng(seed)
    W, I, L = c["hidden_size"], c["intermediate_size"], c["num_hidden_layers"]

    def n(*shape, mean=0.0):
        return (mean + rng.standard_normal(shape) * std).astype(np.float16).astype(np.float32)

    p = {"embeddings.word_embeddings.weight": n(c["vocab_size"], W),
         "embeddings.position_embeddings.weight": n(c["max_position_embeddings"], W),
         "embeddings.token_type_embeddings.weight": n(c["type_vocab_size"], W),
         "embeddings.LayerNorm.weight": n(W, mean=1.0), "embeddings.LayerNorm.bias": n(W)}
    for l in range(L):
        b = "encoder.layer.%d." % l
        for name, (o, i) in (("attention.self.query", (W, W)), ("attention.self.key", (W, W)),
                             ("attention.self.value", (W, W)), ("attention.output.dense", (W, W)),
                             ("intermediate.dense", (I, W)), ("output.dense", (W, I))):
            p[b + name + ".weight"] = n(o, i)
            p[b + name + ".bias"] = n(o)
        for name in ("attention.output.LayerNorm", "output.LayerNorm"):
            p[b + name + ".weight"] = n(W, mean=1.0)
            p[b + name + ".bias"] = n(W)
    return p


def _layer_norm(x, g, b, eps):
    c = x - x.mean(axis=-1, keepdims=True)
    return c / np.sqrt(np.mean(c * c, axis=-1, keepdims=True) + eps) * g + b


def _gelu_erf(x):
    try:
        from scipy.special import erf
    except ImportError:  # pragma: no cover - scipy is present in the supported environments
        erf = np.vectorize(math.erf, otypes=[F64])
    return 0.5 * x * (1.0 + erf(x / math.sqrt(2.0)))


def forward(params, token_ids, attention_mask, token_type_ids=None, position_ids=None, policy="fp64", config=None,
            keep=False):
    """Sentence embeddings [B, hidden] (float64) of token_ids [B, S] under `policy` ("fp64" or "half"); keep=True
    also returns the last hidden rows [B, S, hidden]."""
    if policy not in ("fp64", "half"):
        raise ValueError("policy fp64 or half")
    c = dict(MINILM_L6, **(config or {}))
    W, H, L, eps = c["hidden_size"], c["num_attention_heads"], c["num_hidden_layers"], c["layer_norm_eps"]
    hw = W // H
    ids = np.asarray(token_ids, np.int64)
    B, S = ids.shape
    mask = np.asarray(attention_mask, np.int64).reshape(B, S)
    types = np.zeros_like(ids) if token_type_ids is None else np.asarray(token_type_ids, np.int64)
    pos = np.broadcast_to(np.arange(S), (B, S)) if position_ids is None else np.asarray(position_ids, np.int64)
    if not np.isin(mask, [0, 1]).all() or not mask.any(axis=1).all():
        raise ValueError("refused: 0/1 mask with at least one valid token per sequence required")
    P = {k: np.asarray(v, F64) for k, v in params.items()}
    half = policy == "half"

    def linear(x, prefix):
        w = P[prefix + ".weight"]
        if half:
            x, w = _f16(x), _f16(w)
        return x @ w.T + P[prefix + ".bias"]

    x = P["embeddings.word_embeddings.weight"][ids] + P["embeddings.position_embeddings.weight"][pos] + \
        P["embeddings.token_type_embeddings.weight"][types]
    x = _layer_norm(x, P["embeddings.LayerNorm.weight"], P["embeddings.LayerNorm.bias"], eps)
    keymask = mask[:, None, None, :] == 1                      # [B, 1, 1, S]
    for l in range(L):
        b = "encoder.layer.%d." % l
        q, k, v = (linear(x, b + "attention.self." + n).reshape(B, S, H, hw).transpose(0, 2, 1, 3)
                   for n in ("query", "key", "value"))
        s = (q @ k.transpose(0, 1, 3, 2)) * (1.0 / math.sqrt(hw))
        s = np.where(keymask, s, -np.inf)
        e = np.exp(s - s.max(axis=-1, keepdims=True))
        ctx = ((e / e.sum(axis=-1, keepdims=True)) @ v).transpose(0, 2, 1, 3).reshape(B, S, W)
        x = _layer_norm(linear(ctx, b + "attention.output.dense") + x, P[b + "attention.output.LayerNorm.weight"],
                        P[b + "attention.output.LayerNorm.bias"], eps)
        u = _gelu_erf(linear(x, b + "intermediate.dense"))
        x = _layer_norm(linear(u, b + "output.dense") + x, P[b + "output.LayerNorm.weight"],
                        P[b + "output.LayerNorm.bias"], eps)
    m = mask[:, :, None].astype(F64)
    mean = (x * m).sum(axis=1) / np.maximum(m.sum(axis=1), 1e-9)
    emb = mean / np.maximum(np.linalg.norm(mean, axis=-1, keepdims=True), 1e-12)
    return (emb, x) if keep else emb


def within_bound(got, ref_half):
    """The reference's policy bound |got - ref| <= 2e-4 (1 + |ref|) (g17inferencereference.py:155)."""
    got, ref_half = np.asarray(got, F64), np.asarray(ref_half, F64)
    return np.abs(got - ref_half) <= 2e-4 * (1.0 + np.abs(ref_half))


def cosine(a, b):
    a, b = np.asarray(a, F64).reshape(-1), np.asarray(b, F64).reshape(-1)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))
