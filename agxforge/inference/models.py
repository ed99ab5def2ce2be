"""The decoder shapes the layer builder takes (the reference's agxforge/inference/models.py:26-54 Model records).

    QWEN25_05B      Qwen2.5-0.5B-shaped: 24 layers, d 896, 14 Q / 2 KV heads of 64, FFN 4864, vocab 151,936,
                    qkv bias, tied embeddings (the head is the 4-bit quantisation of the fp16 embedding table),
                    RMSNorm eps 1e-6, RoPE theta 1e6
    INTERNLM25_18B  InternLM2.5-1.8B-shaped: 24 layers, d 2048, 16 Q / 8 KV heads of 128, FFN 8192, vocab 92,544,
                    RoPE theta 1e6 (models.py:42-44: the reference's INTERNLM2 record, eps 1e-5)
    INTERNLM25_7B   InternLM2.5-7B-shaped: 32 layers, d 4096, 32 Q / 8 KV heads of 128, FFN 14336, vocab 92,544
    QWEN3_06B / QWEN3_8B    the Qwen3 family: QK-norm (a per-head RMSNorm of q and k before RoPE), tied head on 0.6B

A record's fields are the upper-case shape attributes the reference's assembler reads (D_MODEL, LAYERS, HEADS,
KV_HEADS, HEAD_DIM, FFN, VOCAB, ROPE_THETA, EPS), plus QKV_BIAS, TIED and QK_NORM.
"""
from __future__ import annotations

import dataclasses


@dataclasses.dataclass(frozen=True)
class Model:
    NAME: str
    D_MODEL: int
    LAYERS: int
    HEADS: int
    KV_HEADS: int
    HEAD_DIM: int
    FFN: int
    VOCAB: int
    ROPE_THETA: float = 1e6
    EPS: float = 1e-6
    QKV_BIAS: bool = False
    TIED: bool = False
    QK_NORM: bool = False

    @property
    def QKV(self):
        return (self.HEADS + 2 * self.KV_HEADS) * self.HEAD_DIM

    def matrices(self):
        """(role, N, K) of every quantized matrix of one layer, then the head."""
        d, F = self.D_MODEL, self.FFN
        return [("qkv", self.QKV, d), ("wo", d, self.HEADS * self.HEAD_DIM), ("gate", F, d), ("up", F, d),
                ("down", d, F)]

    def weight_bytes(self, bits, group=64):
        """Algorithmic bytes of every pack: fields + one 16-bit scale and bias per group (all layers and the head)."""
        per = sum(n * k * bits // 8 + (n * k // group) * 4 for _, n, k in self.matrices())
        head = self.VOCAB * self.D_MODEL * bits // 8 + (self.VOCAB * self.D_MODEL // group) * 4
        return self.LAYERS * per + head

    def kv_bytes_per_position(self):
        """K and V bytes one position adds over every layer (fp16)."""
        return self.LAYERS * 2 * self.KV_HEADS * self.HEAD_DIM * 2

    def replace(self, **kw):
        return dataclasses.replace(self, **kw)


QWEN25_05B = Model("qwen2.5-0.5b", 896, 24, 14, 2, 64, 4864, 151936, 1e6, 1e-6, QKV_BIAS=True, TIED=True)
INTERNLM25_18B = Model("internlm2.5-1.8b", 2048, 24, 16, 8, 128, 8192, 92544, 1e6, 1e-5)
INTERNLM25_7B = Model("internlm2.5-7b", 4096, 32, 32, 8, 128, 14336, 92544, 1e6, 1e-5)

# Qwen3 (the reference's second family, agxforge/inference/models.py:49-64): QK-norm before RoPE, no qkv bias
QWEN3_06B = Model("qwen3-0.6b", 1024, 28, 16, 8, 128, 3072, 151936, 1e6, 1e-6, TIED=True, QK_NORM=True)
QWEN3_8B = Model("qwen3-8b", 4096, 36, 32, 8, 128, 12288, 151936, 1e6, 1e-6, QK_NORM=True)
INTERNLM2 = INTERNLM25_18B      # the reference's name for the InternLM2.5-1.8B record (models.py:42-44)
QWEN3 = {m.NAME: m for m in (QWEN3_06B, QWEN3_8B)}

MODELS = {m.NAME: m for m in (QWEN25_05B, INTERNLM25_18B, INTERNLM25_7B, QWEN3_06B, QWEN3_8B)}


def qwen3(name="qwen3-0.6b"):
    """The Qwen3 record `name` (the reference's qwen3(), models.py:58-64)."""
    if name not in QWEN3:
        raise ValueError("unknown Qwen3 model %r (known: %s)" % (name, ", ".join(sorted(QWEN3))))
    return QWEN3[name]


def get(name):
    if name not in MODELS:
        raise ValueError("unknown model %r (known: %s)" % (name, ", ".join(sorted(MODELS))))
    return MODELS[name]
