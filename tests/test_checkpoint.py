"""Checkpoint import on the CPU (agxforge.inference.checkpoint): the strict safetensors header validation of the
reference (agxforge/g17/inferencegraph.py:45-89) on well-formed and malformed synthetic files, the bounded reader's
refusal of a file that changes while open, the wqkv per-KV-group row permutation (tools/g17q4graph.py:69-74), the
w1 || w3 concatenation (agxforge/inference/assemble.py:26-30), and a whole MLX-format model loaded back into the layer
builder's weights exactly as written."""
import json
import os

import numpy as np
import pytest

from agxforge.inference import checkpoint as CK
from agxforge.inference import models
from oracle import pack as P
from tests import safetensors_io as ST

TINY = models.Model("tiny", 128, 2, 4, 2, 64, 256, 512, 1e6, 1e-5)


def _valid(tmp_path, **kw):
    path = tmp_path / "ok.safetensors"
    ST.write(path, {"a": np.arange(6, dtype=np.float32).reshape(2, 3), "b": np.ones(4, np.uint16)}, **kw)
    return path


def test_header_accepts_a_wellformed_file(tmp_path):
    path = _valid(tmp_path, metadata={"format": "mlx"})
    with CK.Reader(path) as r:
        assert r.names() == ["a", "b"] and r.metadata == {"format": "mlx"}
        assert np.array_equal(r.tensor("a"), np.arange(6, dtype=np.float32).reshape(2, 3))
        assert r.parameters["b"].dtype == "BF16" and r.tensor("b").dtype == np.uint16


def _raw(head):
    return json.dumps(head).encode()


@pytest.mark.parametrize("case,exc", [
    ("duplicate", CK.InvalidCheckpoint), ("extra_field", CK.InvalidCheckpoint), ("dtype", CK.Unsupported),
    ("shape", CK.InvalidCheckpoint), ("extent", CK.InvalidCheckpoint), ("hole", CK.InvalidCheckpoint),
    ("overlap", CK.InvalidCheckpoint), ("metadata", CK.InvalidCheckpoint), ("json", CK.InvalidCheckpoint),
    ("not_mapping", CK.InvalidCheckpoint), ("offsets", CK.InvalidCheckpoint), ("length", CK.InvalidCheckpoint)])
def test_header_refusals(case, exc):
    good = {"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]},
            "b": {"dtype": "F16", "shape": [4], "data_offsets": [8, 16]}}
    raw, total = None, None
    if case == "duplicate":
        raw = b'{"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]}, ' \
              b'"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]}}'
        total = 8 + len(raw) + 8
    elif case == "extra_field":
        good["a"]["extra"] = 1
    elif case == "dtype":
        good["a"]["dtype"] = "F8_E4M3"
    elif case == "shape":
        good["a"]["shape"] = [0]
    elif case == "extent":
        good["a"]["data_offsets"] = [0, 12]
    elif case == "hole":
        good["b"]["data_offsets"] = [12, 20]
    elif case == "overlap":
        good["b"]["data_offsets"] = [4, 12]
    elif case == "metadata":
        good["__metadata__"] = {"k": 3}
    elif case == "json":
        raw = b"{not json"
        total = 8 + len(raw)
    elif case == "not_mapping":
        raw = b"[1, 2]"
        total = 8 + len(raw)
    elif case == "offsets":
        good["a"]["data_offsets"] = [0, -8]
    if raw is None:
        raw = _raw(good)
        total = 8 + len(raw) + 16 + (8 if case == "length" else 0)
    with pytest.raises(exc):
        CK.checkpoint_header(raw, file_bytes=total)


def test_header_size_limits():
    with pytest.raises(CK.InvalidCheckpoint):
        CK.checkpoint_header(b"", file_bytes=8)
    with pytest.raises(CK.InvalidCheckpoint):
        CK.checkpoint_header(b"{}", file_bytes=3)


def test_reader_refuses_a_file_changed_while_open(tmp_path):
    path = _valid(tmp_path)
    r = CK.Reader(path)
    try:
        with open(path, "ab") as f:      # the file grows behind the reader's back
            f.write(b"\0" * 16)
        with pytest.raises(ValueError, match="changed"):
            r.tensor("a")
    finally:
        r.close()


def test_reader_refuses_truncation_and_symlinks(tmp_path):
    path = _valid(tmp_path)
    data = open(path, "rb").read()
    short = tmp_path / "short.safetensors"
    short.write_bytes(data[:-4])
    with pytest.raises(CK.InvalidCheckpoint):
        CK.Reader(short)
    link = tmp_path / "link.safetensors"
    os.symlink(path, link)
    with pytest.raises(OSError):
        CK.Reader(link)


def test_qkv_row_permutation():
    H, KVH, hd = 16, 8, 4
    perm = CK.qkv_rows(H, KVH, hd)
    G = H // KVH
    # the checkpoint's rows: per KV group g: q heads gG .. gG+G-1, k g, v g
    ck = []
    for g in range(KVH):
        ck += [("q", g * G + i) for i in range(G)] + [("k", g), ("v", g)]
    rows = [ck[r // hd] for r in perm]
    want = [("q", h) for h in range(H)] + [("k", g) for g in range(KVH)] + [("v", g) for g in range(KVH)]
    assert rows[::hd] == want
    assert sorted(perm.tolist()) == list(range((H + 2 * KVH) * hd))


def _mlx_checkpoint(path, shape, bits, seed=0, quant_embed=True):
    """A synthetic MLX-format checkpoint of `shape` (bf16 scale and bias patterns, wqkv in the per-group order) and
    the logical packs it holds."""
    S = shape
    rng = np.random.default_rng(seed)

    def q(n, k):
        W = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
        a, s, b, _ = P.quantize(W, bits, scale_dtype="bf16")
        return a, s, b
    t, logical = {}, {}
    inv = np.argsort(CK.qkv_rows(S.HEADS, S.KV_HEADS, S.HEAD_DIM))
    for l in range(S.LAYERS):
        p = "model.layers.%d." % l
        logical[(l, "qkv")] = q(S.QKV, S.D_MODEL)
        ck = [x[inv] for x in logical[(l, "qkv")]]
        for name, val in (("attention.wqkv", ck), ("attention.wo", q(S.D_MODEL, S.HEADS * S.HEAD_DIM)),
                          ("feed_forward.w1", q(S.FFN, S.D_MODEL)), ("feed_forward.w3", q(S.FFN, S.D_MODEL)),
                          ("feed_forward.w2", q(S.D_MODEL, S.FFN))):
            for suf, a in zip((".weight", ".scales", ".biases"), val):
                t[p + name + suf] = a
            logical[(l, {"attention.wqkv": "qkv", "attention.wo": "wo", "feed_forward.w1": "gate",
                         "feed_forward.w3": "up", "feed_forward.w2": "down"}[name])] = tuple(val) \
                if name != "attention.wqkv" else logical[(l, "qkv")]
        g1 = (1 + 0.1 * rng.standard_normal(S.D_MODEL)).astype(np.float32)
        g2 = (1 + 0.1 * rng.standard_normal(S.D_MODEL)).astype(np.float32)
        t[p + "attention_norm.weight"] = CK.f32_to_bf16(g1)
        t[p + "ffn_norm.weight"] = CK.f32_to_bf16(g2)
        logical[(l, "attn_gain")] = CK.bf16_to_f32(t[p + "attention_norm.weight"]).astype(np.float16)
        logical[(l, "ffn_gain")] = CK.bf16_to_f32(t[p + "ffn_norm.weight"]).astype(np.float16)
    t["model.norm.weight"] = CK.f32_to_bf16(np.ones(S.D_MODEL, np.float32))
    logical["final_gain"] = np.ones(S.D_MODEL, np.float16)
    for suf, a in zip((".weight", ".scales", ".biases"), q(S.VOCAB, S.D_MODEL)):
        t["output" + suf] = a
    logical[(None, "head")] = (t["output.weight"], t["output.scales"], t["output.biases"])
    if quant_embed:
        e = q(S.VOCAB, S.D_MODEL)
        for suf, a in zip((".weight", ".scales", ".biases"), e):
            t["model.tok_embeddings" + suf] = a
        logical["embed"] = CK.dequant_embedding(*e, bits, S.D_MODEL)
    else:
        emb = (rng.standard_normal((S.VOCAB, S.D_MODEL)) * 0.02).astype(np.float16)
        t["model.tok_embeddings.weight"] = emb
        logical["embed"] = emb
    # two shards
    names = list(t)
    half = len(names) // 2
    ST.write(path + ".0.safetensors", {n: t[n] for n in names[:half]}, metadata={"format": "mlx"})
    ST.write(path + ".1.safetensors", {n: t[n] for n in names[half:]})
    return [path + ".0.safetensors", path + ".1.safetensors"], logical


@pytest.mark.parametrize("bits", [4, 8])
def test_load_mlx_model_roundtrip(tmp_path, bits):
    paths, logical = _mlx_checkpoint(str(tmp_path / "m"), TINY, bits)
    W, sdt = CK.load(paths, TINY, bits)
    assert sdt == "bf16"
    assert set(W) == set(logical)
    for k, v in logical.items():
        got = W[k]
        if isinstance(v, tuple):
            assert all(np.array_equal(a, b) for a, b in zip(got, v)), k
        else:
            assert np.array_equal(got.view(np.uint16), v.view(np.uint16)), k
    fused = CK.ffn_concat(W, 1)
    assert np.array_equal(fused[0][:TINY.FFN], W[(1, "gate")][0])
    assert np.array_equal(fused[1][TINY.FFN:], W[(1, "up")][1])


def test_load_refuses_mismatched_shapes(tmp_path):
    paths, _ = _mlx_checkpoint(str(tmp_path / "m"), TINY, 4)
    with pytest.raises(CK.InvalidCheckpoint):
        CK.load(paths, TINY.replace(D_MODEL=256), 4)
    with pytest.raises(CK.InvalidCheckpoint):
        CK.load(paths, TINY, 8)                       # 4-bit words read as 8-bit
    with pytest.raises(CK.Unsupported):
        CK.load(paths, TINY, 3)
    with pytest.raises(CK.InvalidCheckpoint, match="missing"):
        CK.load(paths[:1], TINY, 4)


def test_dequant_embedding_matches_the_formula():
    rng = np.random.default_rng(3)
    W = (rng.standard_normal((32, 128)) * 0.05).astype(np.float32)
    a, s, b, q = P.quantize(W, 4, scale_dtype="bf16")
    got = CK.dequant_embedding(a, s, b, 4, 128)
    s32 = CK.bf16_to_f32(s)
    b32 = CK.bf16_to_f32(b)
    w = (q.reshape(32, 2, 64).astype(np.float32) * s32[..., None] + b32[..., None]).reshape(32, 128)
    want = CK.bf16_to_f32(CK.f32_to_bf16(w)).astype(np.float16)
    assert np.array_equal(got.view(np.uint16), want.view(np.uint16))
