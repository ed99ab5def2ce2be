"""Checkpoint import: MLX-format quantized packs read from safetensors files into the layer builder's weights (the
reference's checkpoint path: agxforge/g17/inferencegraph.py:45-89 checkpoint_header, tools/g17checkpoint.py's bounded
reader, and tools/g17q4graph.py:69-112 / agxforge/inference/assemble.py:26-30 for the MLX layout).

    checkpoint_header(raw, file_bytes)  the strict header validation of inferencegraph.py:45-89: the header is 1 B to
                                        4 MiB of JSON with unique keys, `__metadata__` string pairs, every tensor record
                                        exactly {dtype, shape, data_offsets}, the byte extent equal to shape x element
                                        size, the payload covered contiguously (no hole, no overlap) and ending at the
                                        file's last byte; returns {name: Parameter}. Malformed input raises
                                        InvalidCheckpoint, an unknown dtype Unsupported (both ValueError)
    Reader(path)                        one opened file, validated once; tensors read by offset (os.pread, bounded
                                        chunks) from that inode, with its size and times checked around every read
                                        (tools/g17checkpoint.py:54-109), as numpy arrays
    qkv_rows(heads, kv_heads, head_dim) the row order that takes the checkpoint's per-KV-group wqkv packing
                                        [q g*G .. q g*G+G-1, k g, v g] to q heads | k heads | v heads (g17q4graph.py:69-74)
    load(paths, model, bits)            the weights dict assemble.build(weights=...) takes, from mlx_lm.convert -q
                                        output (InternLM2 names): packs as (packed uint32, scales, biases) with bf16
                                        scale and bias patterns, wqkv rows permuted, norm gains fp16, and the embedding
                                        as the reference keeps it: the dequantised table stored fp16 (its import calls
                                        mlx.dequantize, whose result takes the scales' bf16 type; here w = s q + b in
                                        fp32, rounded once to bf16, then to fp16)
    ffn_concat(weights, layer)          the reference's fused FFN pack: w1 rows then w3 rows (assemble.py:26-30), the
                                        qmv_swiglu_layout operand (the layer builder interleaves gate and up itself)

Only rows move: a row permutation carries each row's scales and biases with it, so no value changes. The file's
contents are not trusted beyond its header's consistency: a tensor read outside the validated extents, a file that
changes while open, or a shape that does not match the model is refused.
"""
from __future__ import annotations

import json
import math
import os
import stat
from dataclasses import dataclass

import numpy as np

CHUNK = 1024 * 1024
HEADER_MAX = 4 * 1024 * 1024
# safetensors element types this reader admits: the reference's set (inferencegraph.py:20) plus the 32-bit words and
# bytes of quantized packs
ELEMENT_BYTES = {"F32": 4, "F16": 2, "BF16": 2, "I32": 4, "I64": 8, "U32": 4, "U8": 1}
NUMPY = {"F32": np.float32, "F16": np.float16, "BF16": np.uint16, "I32": np.int32, "I64": np.int64,
         "U32": np.uint32, "U8": np.uint8}


class Unsupported(ValueError):
    """A recognised checkpoint feature outside this importer's domain."""


class InvalidCheckpoint(ValueError):
    """Malformed or contradictory checkpoint metadata."""


@dataclass(frozen=True)
class Parameter:
    name: str
    dtype: str
    shape: tuple
    begin: int
    end: int

    @property
    def bytes(self):
        return self.end - self.begin


def _unique(pairs):
    out = {}
    for k, v in pairs:
        if k in out:
            raise InvalidCheckpoint("duplicate JSON key: " + k)
        out[k] = v
    return out


def checkpoint_header(raw, *, file_bytes):
    """Validate a safetensors header against the exact whole-file length (inferencegraph.py:45-89)."""
    if not isinstance(raw, bytes) or not 1 <= len(raw) <= HEADER_MAX:
        raise InvalidCheckpoint("header must be 1..4 MiB of bytes")
    if type(file_bytes) is not int or file_bytes < 8 + len(raw):
        raise InvalidCheckpoint("invalid checkpoint byte length")
    try:
        data = json.loads(raw, object_pairs_hook=_unique)
    except (UnicodeDecodeError, json.JSONDecodeError) as exc:
        raise InvalidCheckpoint("invalid header JSON") from exc
    if not isinstance(data, dict):
        raise InvalidCheckpoint("header must be a mapping")
    metadata = data.pop("__metadata__", {})
    if not isinstance(metadata, dict) or any(not isinstance(k, str) or not isinstance(v, str)
                                             for k, v in metadata.items()):
        raise InvalidCheckpoint("metadata must contain string pairs")
    params = {}
    for name, spec in data.items():
        if not name or not isinstance(spec, dict) or set(spec) != {"dtype", "shape", "data_offsets"}:
            raise InvalidCheckpoint("invalid tensor record: " + str(name))
        dtype, shape, offsets = spec["dtype"], spec["shape"], spec["data_offsets"]
        if not isinstance(dtype, str) or dtype not in ELEMENT_BYTES:
            raise Unsupported("refused: checkpoint dtype " + repr(dtype))
        if not isinstance(shape, list) or len(shape) > 8 or any(type(d) is not int or d <= 0 for d in shape):
            raise InvalidCheckpoint("invalid shape: " + name)
        if not isinstance(offsets, list) or len(offsets) != 2 or any(type(d) is not int or d < 0 for d in offsets):
            raise InvalidCheckpoint("invalid offsets: " + name)
        begin, end = offsets
        if end - begin != math.prod(shape) * ELEMENT_BYTES[dtype]:
            raise InvalidCheckpoint("shape/dtype/byte extent disagreement: " + name)
        params[name] = Parameter(name, dtype, tuple(shape), begin, end)
    cursor = 0
    for p in sorted(params.values(), key=lambda p: (p.begin, p.end)):
        if p.begin != cursor:
            raise InvalidCheckpoint("payload overlap or hole: " + p.name)
        cursor = p.end
    if 8 + len(raw) + cursor != file_bytes:
        raise InvalidCheckpoint("payload extent does not match whole file")
    return params


def _identity(st):
    return st.st_size, st.st_mtime_ns, st.st_ctime_ns


class Reader:
    """One safetensors file opened once (no symlink followed), its header validated against the file's length, its
    tensors read by offset from that inode; a file that changes while open is refused (tools/g17checkpoint.py:54-109)."""

    def __init__(self, path):
        self.path = os.fspath(path)
        self.fd = os.open(self.path, os.O_RDONLY | getattr(os, "O_NOFOLLOW", 0))
        try:
            st = os.fstat(self.fd)
            if not stat.S_ISREG(st.st_mode):
                raise InvalidCheckpoint("not a regular file: " + self.path)
            self.identity = _identity(st)
            head = os.pread(self.fd, 8, 0)
            if len(head) != 8:
                raise InvalidCheckpoint("truncated header length")
            n = int.from_bytes(head, "little")
            if not 1 <= n <= HEADER_MAX:
                raise InvalidCheckpoint("header must be 1..4 MiB of bytes")
            raw = os.pread(self.fd, n, 8)
            if len(raw) != n:
                raise InvalidCheckpoint("truncated header")
            self.header_bytes = n
            self.parameters = checkpoint_header(raw, file_bytes=st.st_size)
            self.metadata = json.loads(raw).get("__metadata__", {})
        except BaseException:
            os.close(self.fd)
            raise

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def close(self):
        if self.fd is not None:
            os.close(self.fd)
            self.fd = None

    def check(self):
        if self.fd is None:
            raise ValueError("checkpoint reader is closed")
        if _identity(os.fstat(self.fd)) != self.identity:
            raise ValueError("checkpoint changed while open")

    def names(self):
        return sorted(self.parameters)

    def tensor(self, name):
        """The tensor as a numpy array of its stored type (BF16 as uint16 bit patterns)."""
        if name not in self.parameters:
            raise KeyError("no tensor %r in %s" % (name, self.path))
        self.check()
        p = self.parameters[name]
        out = bytearray(p.bytes)
        off = 8 + self.header_bytes + p.begin
        got = 0
        while got < p.bytes:
            blk = os.pread(self.fd, min(CHUNK, p.bytes - got), off + got)
            if not blk:
                raise ValueError("checkpoint truncated during tensor read")
            out[got:got + len(blk)] = blk
            got += len(blk)
        self.check()
        return np.frombuffer(bytes(out), NUMPY[p.dtype]).reshape(p.shape)


def qkv_rows(heads, kv_heads, head_dim):
    """new row -> checkpoint row of the packed wqkv: the checkpoint holds, per KV group g, the group's G query heads,
    then k head g, then v head g; the layer builder wants every q head, then every k head, then every v head."""
    if heads % kv_heads:
        raise ValueError("qkv_rows: heads a multiple of kv_heads")
    G = heads // kv_heads
    old = np.arange((heads + 2 * kv_heads) * head_dim).reshape(kv_heads, G + 2, head_dim)
    q = old[:, :G].reshape(-1)
    return np.concatenate([q, old[:, G].reshape(-1), old[:, G + 1].reshape(-1)])


def bf16_to_f32(u16):
    return (np.asarray(u16, np.uint32) << 16).view(np.float32)


def f32_to_bf16(x):
    """Round-to-nearest-even fp32 -> bf16 bit patterns."""
    u = np.asarray(x, np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def dequant_embedding(packed, scales, biases, bits, dim):
    """The embedding table of a quantized checkpoint, dequantised and stored fp16 as the reference's import keeps it
    (g17q4graph.py:107-109): w = s q + b in fp32, rounded once to bf16 (the scales' type, the type mlx.dequantize
    returns), then to fp16."""
    V = packed.shape[0]
    per = 32 // bits
    sh = (bits * np.arange(per)).astype(np.uint32)
    out = np.empty((V, dim), np.float16)
    step = max(1, (1 << 22) // dim)
    for r0 in range(0, V, step):
        w = np.asarray(packed[r0:r0 + step], np.uint32)
        q = ((w[:, :, None] >> sh) & np.uint32((1 << bits) - 1)).reshape(w.shape[0], dim).astype(np.float32)
        s = bf16_to_f32(scales[r0:r0 + step])
        b = bf16_to_f32(biases[r0:r0 + step])
        x = (q.reshape(w.shape[0], dim // 64, 64) * s[..., None] + b[..., None]).reshape(w.shape[0], dim)
        out[r0:r0 + step] = bf16_to_f32(f32_to_bf16(x)).astype(np.float16)
    return out


def _gain(a):
    a = np.asarray(a)
    if a.dtype == np.uint16:                    # BF16 patterns
        return bf16_to_f32(a).astype(np.float16)
    return a.astype(np.float16)


class _Files:
    """Several safetensors shards as one name space (every name in exactly one file)."""

    def __init__(self, paths):
        self.readers = [Reader(p) for p in paths]
        self.where = {}
        for r in self.readers:
            for n in r.parameters:
                if n in self.where:
                    raise InvalidCheckpoint("tensor %r in two shards" % n)
                self.where[n] = r

    def tensor(self, name):
        if name not in self.where:
            raise InvalidCheckpoint("missing tensor: " + name)
        return self.where[name].tensor(name)

    def close(self):
        for r in self.readers:
            r.close()


def load(paths, model, bits, group=64):
    """Weights for assemble.build(weights=...) from MLX-format shards (InternLM2 names: model.layers.{l}.attention.
    {wqkv,wo}, feed_forward.{w1,w3,w2} as {weight, scales, biases}; attention_norm / ffn_norm / model.norm weights;
    output; model.tok_embeddings quantized or plain). `model` is an agxforge.inference.models.Model (the shapes are
    checked against every tensor). Returns the dict and the build config's scale_dtype ("bf16")."""
    if isinstance(paths, (str, os.PathLike)):
        paths = [paths]
    if bits not in (4, 8) or group != 64:
        raise Unsupported("refused: %d-bit group-%d packs (4 or 8 bits, group 64)" % (bits, group))
    S = model
    f = _Files(paths)
    try:
        def trio(prefix, n, k):
            w, s, b = (f.tensor(prefix + x) for x in (".weight", ".scales", ".biases"))
            if w.dtype != np.uint32 or w.shape != (n, k * bits // 32):
                raise InvalidCheckpoint("%s.weight: uint32 [%d, %d] expected, %s %s found" % (
                    prefix, n, k * bits // 32, w.dtype, w.shape))
            for x, nm in ((s, "scales"), (b, "biases")):
                if x.dtype != np.uint16 or x.shape != (n, k // group):
                    raise InvalidCheckpoint("%s.%s: bf16 [%d, %d] expected" % (prefix, nm, n, k // group))
            return np.ascontiguousarray(w), np.ascontiguousarray(s), np.ascontiguousarray(b)

        W = {}
        perm = qkv_rows(S.HEADS, S.KV_HEADS, S.HEAD_DIM)
        d, F, hd = S.D_MODEL, S.FFN, S.HEADS * S.HEAD_DIM
        for l in range(S.LAYERS):
            p = "model.layers.%d." % l
            w, s, b = trio(p + "attention.wqkv", S.QKV, d)
            W[(l, "qkv")] = (w[perm], s[perm], b[perm])
            W[(l, "wo")] = trio(p + "attention.wo", d, hd)
            W[(l, "gate")] = trio(p + "feed_forward.w1", F, d)
            W[(l, "up")] = trio(p + "feed_forward.w3", F, d)
            W[(l, "down")] = trio(p + "feed_forward.w2", d, F)
            W[(l, "attn_gain")] = _gain(f.tensor(p + "attention_norm.weight"))
            W[(l, "ffn_gain")] = _gain(f.tensor(p + "ffn_norm.weight"))
            for key in ((l, "attn_gain"), (l, "ffn_gain")):
                if W[key].shape != (d,):
                    raise InvalidCheckpoint("norm gain of layer %d: [%d] expected" % (l, d))
        W["final_gain"] = _gain(f.tensor("model.norm.weight"))
        if W["final_gain"].shape != (d,):
            raise InvalidCheckpoint("model.norm.weight: [%d] expected" % d)
        W[(None, "head")] = trio("output", S.VOCAB, d)
        if "model.tok_embeddings.scales" in f.where:
            e, es, eb = trio("model.tok_embeddings", S.VOCAB, d)
            W["embed"] = dequant_embedding(e, es, eb, bits, d)
        else:
            e = f.tensor("model.tok_embeddings.weight")
            if e.shape != (S.VOCAB, d):
                raise InvalidCheckpoint("model.tok_embeddings.weight: [%d, %d] expected" % (S.VOCAB, d))
            W["embed"] = _gain(e)
        return W, "bf16"
    finally:
        f.close()


def ffn_concat(weights, layer):
    """The reference's fused FFN pack of one layer: w1 (gate) rows then w3 (up) rows, scales and biases alike
    (assemble.py:26-30) — the operand of qmv_swiglu_layout / qmv_swiglu_reference."""
    g, u = weights[(layer, "gate")], weights[(layer, "up")]
    return tuple(np.concatenate([a, b]) for a, b in zip(g, u))
