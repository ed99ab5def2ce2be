"""The BERT sentence encoder (MiniLM-L6 shape) on the B200: the reference's complete-encoder path
(agxforge/g17/inferencegraph.py:208-289 ``import_graph`` with sentence pooling; its FP64 reference
tools/g17inferencereference.py:18-99 ``graph_reference``), batched over padded sequences.

    Encoder(config, max_batch=32, max_seq=128)   the device encoder for a BERT config dict (the checkpoint's
                                                 config.json fields; refused like the reference's ``profile``)
    Encoder.load(parameters)                     parameters by checkpoint name (numpy or torch; stored fp16)
    Encoder.synthetic(config, seed)              seeded random-init parameters generated on the device
    Encoder.forward(inputs)                      inputs {"token_ids", "attention_mask"[, "token_type_ids",
                                                 "position_ids"]} of shape [batch, seq] (or [seq]) -> sentence
                                                 embeddings float32 [batch, hidden] (mean over the valid rows,
                                                 L2-normalised)
    Encoder.forward_device(ids, mask, ...)       the same on device tensors, enqueued on the library's stream

Linear layers run on the tensor cores with fp16 operands and fp32 accumulation (the reference's half-transport
policy); LayerNorm, GELU (erf), softmax and pooling are fp32. Inputs outside their domain raise ValueError
("refused: ...") as the reference does. There is no CPU path.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from agxforge_b200 import _native as N

LAYER_PARAMS = {
    "attention.self.query.weight": 5, "attention.self.query.bias": 6,
    "attention.self.key.weight": 7, "attention.self.key.bias": 8,
    "attention.self.value.weight": 9, "attention.self.value.bias": 10,
    "attention.output.dense.weight": 11, "attention.output.dense.bias": 12,
    "attention.output.LayerNorm.weight": 13, "attention.output.LayerNorm.bias": 14,
    "intermediate.dense.weight": 15, "intermediate.dense.bias": 16,
    "output.dense.weight": 17, "output.dense.bias": 18,
    "output.LayerNorm.weight": 19, "output.LayerNorm.bias": 20,
}
EMBED_PARAMS = {
    "embeddings.word_embeddings.weight": 0, "embeddings.position_embeddings.weight": 1,
    "embeddings.token_type_embeddings.weight": 2, "embeddings.LayerNorm.weight": 3, "embeddings.LayerNorm.bias": 4,
}


# BASELINE config 2's shape (sentence-transformers MiniLM-L6: the checkpoint's config.json fields)
MINILM_L6 = dict(model_type="bert", architectures=["BertModel"], hidden_size=384, num_attention_heads=12,
                 intermediate_size=1536, num_hidden_layers=6, vocab_size=30522, max_position_embeddings=512,
                 type_vocab_size=2, layer_norm_eps=1e-12, hidden_act="gelu")


def check_config(config):
    """The reference's admission of a BERT config (agxforge/g17/inferencegraph.py:116-157), plus this encoder's
    shape limits. Returns (hidden, layers, heads, ffn, vocab, max_position, type_vocab, eps)."""
    if not isinstance(config, dict):
        raise ValueError("refused: model config must be a mapping")
    if config.get("model_type") != "bert" or config.get("architectures") != ["BertModel"]:
        raise ValueError("refused: a BertModel config is required")
    if config.get("hidden_act") != "gelu":
        raise ValueError("refused: activation outside the selected architecture")
    if config.get("position_embedding_type", "absolute") != "absolute" or config.get("is_decoder", False) or \
            config.get("add_cross_attention", False):
        raise ValueError("refused: BERT relative positions or decoder/cross attention")
    try:
        v = [int(config[k]) for k in ("hidden_size", "num_hidden_layers", "num_attention_heads", "intermediate_size",
                                      "vocab_size", "max_position_embeddings", "type_vocab_size")]
    except (KeyError, TypeError, ValueError):
        raise ValueError("refused: positive integer config fields required") from None
    if min(v) <= 0:
        raise ValueError("refused: positive integer config fields required")
    eps = config.get("layer_norm_eps")
    if not isinstance(eps, (int, float)) or not eps > 0:
        raise ValueError("refused: positive finite normalization epsilon required")
    W, L, H, F = v[:4]
    if W % H or W // H not in (32, 64) or W % 128 or W > 1024 or F % 64:
        raise ValueError("refused: hidden a multiple of 128 (<= 1024), head width 32 or 64, ffn a multiple of 64")
    return (*v, float(eps))


class Encoder:
    def __init__(self, config, max_batch=32, max_seq=128, device=0):
        import torch
        if not torch.cuda.is_available():
            raise RuntimeError("agxforge needs a CUDA device (B200); none is visible")
        self.config = dict(config)
        W, L, H, F, V, P, T, eps = check_config(self.config)
        self.hidden, self.layers, self.heads, self.ffn, self.vocab = W, L, H, F, V
        self.max_position, self.type_vocab = P, T
        self.max_batch, self.max_seq = int(max_batch), int(max_seq)
        self.device = device
        torch.cuda.set_device(device)
        d = N.EncoderDesc(W, L, H, F, V, P, T, eps, self.max_batch, self.max_seq)
        h = C.c_void_p()
        N.check(N.lib().agxc_encoder_create(N.context(device), C.byref(d), C.byref(h)), "encoder_create")
        self._h = h

    # ---------------------------------------------------------------- parameters
    def _shape(self, name):
        W, F = self.hidden, self.ffn
        if name in EMBED_PARAMS:
            return {"embeddings.word_embeddings.weight": (self.vocab, W),
                    "embeddings.position_embeddings.weight": (self.max_position, W),
                    "embeddings.token_type_embeddings.weight": (self.type_vocab, W)}.get(name, (W,))
        if name.endswith(".weight") and "LayerNorm" not in name:
            if name.startswith("intermediate"):
                return (F, W)
            if name.startswith("output.dense"):
                return (W, F)
            return (W, W)
        return (F,) if name == "intermediate.dense.bias" else (W,)

    def set_param(self, name, value):
        """One parameter by checkpoint name (e.g. encoder.layer.3.attention.self.query.weight), stored as fp16."""
        if name in EMBED_PARAMS:
            layer, which, local = 0, EMBED_PARAMS[name], name
        else:
            parts = name.split(".")
            if len(parts) < 4 or parts[0] != "encoder" or parts[1] != "layer" or not parts[2].isdigit():
                raise ValueError("refused: unknown parameter " + name)
            layer, local = int(parts[2]), ".".join(parts[3:])
            if local not in LAYER_PARAMS or not 0 <= layer < self.layers:
                raise ValueError("refused: unknown parameter " + name)
            which = LAYER_PARAMS[local]
        shape = self._shape(local)
        if hasattr(value, "detach"):
            import torch
            t = value.detach().to(device="cuda:%d" % self.device, dtype=torch.float16).contiguous()
            if tuple(t.shape) != shape:
                raise ValueError("refused: %s has shape %s, expected %s" % (name, tuple(t.shape), shape))
            torch.cuda.synchronize()
            N.check(N.lib().agxc_encoder_set_param(self._h, layer, which, C.c_void_p(t.data_ptr()), t.numel() * 2,
                                                   1), "set_param " + name)
        else:
            a = np.ascontiguousarray(np.asarray(value).astype(np.float16))
            if a.shape != shape:
                raise ValueError("refused: %s has shape %s, expected %s" % (name, a.shape, shape))
            N.check(N.lib().agxc_encoder_set_param(self._h, layer, which, a.ctypes.data_as(C.c_void_p), a.nbytes, 0),
                    "set_param " + name)

    def load(self, parameters):
        """Every parameter of the encoder, by checkpoint name; the pooler and position_ids buffers are ignored (the
        reference's allowed unused tensors, inferencegraph.py:292-296)."""
        want = set(EMBED_PARAMS) | {"encoder.layer.%d.%s" % (l, k) for l in range(self.layers) for k in LAYER_PARAMS}
        missing = want - set(parameters)
        if missing:
            raise ValueError("refused: missing model parameter " + sorted(missing)[0])
        extra = set(parameters) - want - {"embeddings.position_ids", "pooler.dense.weight", "pooler.dense.bias"}
        if extra:
            raise ValueError("refused: unconsumed checkpoint tensor " + sorted(extra)[0])
        for name in sorted(want):
            self.set_param(name, parameters[name])
        return self

    @classmethod
    def synthetic(cls, config, seed=1, std=0.02, **kw):
        """Random-init parameters generated on the device from `seed` (linear weights, biases and embeddings
        N(0, std); LayerNorm gains 1 + N(0, std) and biases N(0, std)); throughput runs."""
        import torch
        enc = cls(config, **kw)
        g = torch.Generator(device="cuda:%d" % enc.device)
        g.manual_seed(int(seed))
        names = sorted(set(EMBED_PARAMS) | {"encoder.layer.%d.%s" % (l, k) for l in range(enc.layers)
                                             for k in LAYER_PARAMS})
        for name in names:
            local = name if name in EMBED_PARAMS else ".".join(name.split(".")[3:])
            shape = enc._shape(local)
            t = torch.randn(shape, generator=g, device="cuda:%d" % enc.device) * std
            if "LayerNorm.weight" in name:
                t += 1.0
            enc.set_param(name, t)
        return enc

    # ---------------------------------------------------------------- forward
    def _inputs(self, inputs):
        if set(inputs) - {"token_ids", "attention_mask", "token_type_ids", "position_ids"} or \
                not {"token_ids", "attention_mask"} <= set(inputs):
            raise ValueError("refused: encoder input inventory (token_ids, attention_mask[, token_type_ids, "
                             "position_ids])")
        ids = np.asarray(inputs["token_ids"])
        if ids.ndim == 1:
            ids = ids[None]
        if ids.ndim != 2:
            raise ValueError("refused: token_ids of shape [batch, seq] or [seq]")
        B, S = ids.shape
        mask = np.asarray(inputs["attention_mask"]).reshape(B, S)
        types = inputs.get("token_type_ids")
        if "position_ids" in inputs and inputs["position_ids"] is not None:
            pos = np.asarray(inputs["position_ids"]).reshape(-1, S)
            if not (pos == np.arange(S)).all():
                raise ValueError("refused: position_ids other than 0 .. seq-1")
        if not np.isin(mask, [0, 1]).all() or not mask.any(axis=1).all():
            raise ValueError("refused: 0/1 mask with at least one valid token required")
        if ids.min() < 0 or ids.max() >= self.vocab:
            raise ValueError("refused: reference index outside domain: token_ids")
        if types is not None:
            types = np.asarray(types).reshape(B, S)
            if types.min() < 0 or types.max() >= self.type_vocab:
                raise ValueError("refused: reference index outside domain: token_type_ids")
            types = np.ascontiguousarray(types, np.int32)
        if not 1 <= B <= self.max_batch or not 1 <= S <= min(self.max_seq, self.max_position):
            raise ValueError("refused: batch 1..%d and seq 1..%d" % (self.max_batch, min(self.max_seq,
                                                                                           self.max_position)))
        return np.ascontiguousarray(ids, np.int32), np.ascontiguousarray(mask, np.int32), types

    def forward(self, inputs, timing=False):
        """Sentence embeddings float32 [batch, hidden]; timing=True also returns {gpu_ms, host_ms, launches}."""
        ids, mask, types = self._inputs(inputs)
        B, S = ids.shape
        out = np.empty((B, self.hidden), np.float32)
        t = N.Timing()
        N.check(N.lib().agxc_encoder_forward(self._h, ids.ctypes.data_as(C.c_void_p), mask.ctypes.data_as(C.c_void_p),
                                             None if types is None else types.ctypes.data_as(C.c_void_p), B, S,
                                             out.ctypes.data_as(C.c_void_p), 0, C.byref(t)), "encoder_forward")
        if timing:
            return out, dict(gpu_ms=t.gpu_ms, host_ms=t.host_ms, launches=t.launches_per_step)
        return out

    def forward_device(self, ids, mask, types=None, out=None):
        """Device tensors int32 [batch, seq] -> out float32 [batch, hidden] (allocated when None), enqueued on the
        library's stream, ordered after torch's current stream (which produced the inputs) and before its later work
        (which reads `out`) with events, no host synchronisation; an id or type outside its table is reported by the
        next synchronising call."""
        import torch
        B, S = ids.shape
        for t in (ids, mask) + ((types,) if types is not None else ()):
            if t.dtype != torch.int32 or not t.is_cuda or not t.is_contiguous() or tuple(t.shape) != (B, S):
                raise ValueError("refused: int32 contiguous device tensors [batch, seq]")
        if out is None:
            out = torch.empty((B, self.hidden), dtype=torch.float32, device=ids.device)
        mine, theirs = N.ctx_stream(self.device), torch.cuda.current_stream(ids.device)
        mine.wait_stream(theirs)
        N.check(N.lib().agxc_encoder_forward(self._h, C.c_void_p(ids.data_ptr()), C.c_void_p(mask.data_ptr()),
                                             None if types is None else C.c_void_p(types.data_ptr()), B, S,
                                             C.c_void_p(out.data_ptr()), 1, None), "encoder_forward")
        for t in (ids, mask, out) + ((types,) if types is not None else ()):
            t.record_stream(mine)  # torch's allocator keeps them until the library's stream is past this forward
        theirs.wait_stream(mine)
        return out

    def replay(self, reps, flush_l2=True):
        """`reps` forwards on the last forward's inputs (resident on the device), L2 flushed before each when
        flush_l2: device ms of the forwards, launches per forward."""
        t = N.Timing()
        N.check(N.lib().agxc_encoder_replay(self._h, int(reps), int(bool(flush_l2)), C.byref(t)), "encoder_replay")
        return dict(gpu_ms=t.gpu_ms, host_ms=t.host_ms, launches=t.launches_per_step)

    def profile(self, batch, seq, reps=3):
        """Per-stage device time (ms summed over `reps` forwards, each launch timed on its own) and launch counts."""
        ms = (C.c_float * 8)()
        n = (C.c_int32 * 8)()
        N.check(N.lib().agxc_encoder_profile(self._h, batch, seq, reps, ms, n), "encoder_profile")
        names = ["embed", "qkv", "attn", "o_proj", "layernorm", "ffn_up", "ffn_down", "pool"]
        return {k: dict(ms=ms[i], launches=n[i]) for i, k in enumerate(names)}

    def close(self):
        h = getattr(self, "_h", None)
        lib = getattr(N, "_lib", None) if N is not None else None
        if h and lib is not None:
            lib.agxc_encoder_free(h)
        self._h = None

    def __del__(self):
        self.close()
