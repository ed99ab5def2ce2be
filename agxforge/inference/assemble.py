"""The layer builder: a decoder's weights, KV cache and decode graph on the B200 (the reference's
agxforge/inference/assemble.py: configure 71-92, build 596-828; its region R and token log 650-669).

    configure(config)           a config dict (or JSON path): {"model": name | shape overrides, "bits", "scale_dtype",
                                "cap", "batch", "seed", "keep_logits", "tp", "tp_rank"}; returns the normalised config
                                (tp > 1: tensor parallel over tp ranks, one process per GPU, torch.distributed
                                initialised; each rank builds its shard of the same seeded weights, see tp.py).
                                configure(deliver, config), the reference's two-argument form, is accepted: the
                                deliver index of compiled G17 bundles has no counterpart and is ignored; the config
                                becomes the module's current one, which build(bits) uses
    build(config, ...)          a DecodeModel: the library's model object with every pack, gain, bias and the
                                embedding set. Synthetic weights are generated on the device from the config's seed
                                (N(0, 0.02) fp32, then the device quantiser), or taken from given reference-format
                                packs (`weights=`, e.g. checkpoint.load). build(bits) (the reference's form) builds the
                                current config at that width; the reference returns (graph.json dict, ops), here the
                                device model is the graph
    simulate(bits, tokens)      the reference's CPU replay of the built graph (assemble.py:934-955) is not part of this
                                package (it has no CPU path); the CPU restatement of the decode step that the tests
                                compare against lives in the repository's oracle package
    DecodeModel.start(b, prompt)  the sequence's prompt in its token log, x = embedding(prompt[0]), q0 = 0
    DecodeModel.decode(steps)     run steps (execute.decode wraps it in the reference's report)

At batch 1..8 the layer is five kernels (RMSNorm + qkv + bias + RoPE + append, split-KV attention + merge, o_proj +
residual, RMSNorm + gate/up + SiLU*mul, down + residual) and the head one (final norm + vocabulary GEMV + argmax +
generation step), chained by programmatic dependent launch in one CUDA graph a step; at 32..256 sequences the
projections are tensor-core GEMMs. At batch 1 on one device the "fused" option runs the whole step as one persistent
kernel instead (each CTA waiting only on the counters of the data it reads).
"""
from __future__ import annotations

import ctypes as C
import json
import os

import numpy as np

from agxforge_b200 import _native as N
from agxforge.inference import models
from agxforge.inference import tp as TP
from agxforge.kernels import qmv as Q

ROLE = {"qkv": N.ROLE_QKV, "wo": N.ROLE_WO, "gate": N.ROLE_GATE, "up": N.ROLE_UP, "down": N.ROLE_DOWN,
        "head": N.ROLE_HEAD}
ROLE_INDEX = {"qkv": 0, "wo": 1, "gate": 2, "up": 3, "down": 4, "head": 5}

DEFAULTS = dict(model="internlm2.5-1.8b", bits=4, scale_dtype="fp16", cap=2048, batch=1, seed=2, keep_logits=False,
                init_std=0.02, embed_std=0.02, bias_std=0.02)


_current = None


def configure(*args):
    """Normalise a config (dict or path of a JSON file): configure(config), or the reference's configure(deliver,
    config) with the deliver index ignored. The result is also the module's current config (for build(bits))."""
    global _current
    if len(args) == 1:
        config = args[0]
    elif len(args) == 2:
        config = args[1]
    else:
        raise TypeError("configure(config) or configure(deliver, config)")
    if isinstance(config, (str, os.PathLike)):
        with open(config) as f:
            config = json.load(f)
    cfg = dict(DEFAULTS)
    cfg.update(config or {})
    shape = cfg["model"]
    if isinstance(shape, str):
        shape = models.get(shape)
    elif isinstance(shape, dict):
        shape = dict(shape)
        base = models.get(shape.pop("base")) if "base" in shape else None
        shape = base.replace(**shape) if base else models.Model(**shape)
    cfg["shape"] = shape
    if cfg["bits"] not in (4, 8):
        raise ValueError("configure: bits 4 or 8")
    if cfg["scale_dtype"] not in Q.SCALE_DTYPES:
        raise ValueError("configure: scale_dtype fp16 or bf16")
    B = int(cfg["batch"])
    if not (1 <= B <= 8 or (32 <= B <= 256 and B % 16 == 0)):
        raise ValueError("configure: batch 1..8 (GEMV step), or 32..256 in steps of 16 (tensor-core GEMM step)")
    cfg["tp"] = int(cfg.get("tp") or 1)
    cfg["tp_rank"] = int(cfg.get("tp_rank") or 0)
    TP.check(shape, cfg["tp"], B)
    if not 0 <= cfg["tp_rank"] < cfg["tp"]:
        raise ValueError("configure: 0 <= tp_rank < tp")
    _current = cfg
    return cfg


def simulate(bits, tokens):
    """The reference's CPU replay (assemble.py:934-955). This package runs only on the device; the CPU restatement
    of the decode step used as the parity oracle is test infrastructure outside it."""
    raise NotImplementedError("simulate: the CPU replay of the decode step is not part of the agxforge package on "
                              "the B200 (no CPU path); the repository's oracle package restates it for the tests")


def _gen(torch, seed, *key):
    g = torch.Generator(device="cuda")
    g.manual_seed((int(seed) * 1000003 + hash_key(*key)) % (2 ** 63))
    return g


def hash_key(*key):
    """A stable integer for a (layer, role) key (seed derivation; Python's hash() is salted per process)."""
    h = 1469598103934665603
    for part in key:
        for ch in str(part).encode():
            h = ((h ^ ch) * 1099511628211) % (2 ** 64)
        h = ((h ^ 0xFF) * 1099511628211) % (2 ** 64)
    return h


FUSED_TRACE_MARKS = 26   # the fused step's trace marks a layer (trace_fused)
# the fused step's cycle-profile regions, in the library's order (profile_fused); "" = unused
FUSED_PROFILE_REGIONS = ["top", "preload", "wait", "act_load", "norm", "rows", "rows_reduce", "qkv_epilogue",
                         "signal", "attn_q", "attn_keys", "attn_merge", "attn_out", "o_merge", "owned", "silu",
                         "head_argmax", "tail", "owned_wait", "rows_wait", "attn_wait", "", "", ""]


class DecodeModel:
    """The device model (owns the library's model object)."""

    def __init__(self, cfg, device=0, tp_id=None):
        import torch
        if not torch.cuda.is_available():
            raise RuntimeError("agxforge needs a CUDA device (B200); none is visible")
        self.cfg = cfg
        self.shape = S = cfg["shape"]
        self.device = device
        self.bits = int(cfg["bits"])
        self.batch = int(cfg["batch"])
        self.cap = int(cfg["cap"])
        d = N.ModelDesc(S.D_MODEL, S.LAYERS, S.HEADS, S.KV_HEADS, S.HEAD_DIM, S.FFN, S.VOCAB, self.bits, 64,
                        Q.SCALE_DTYPES[cfg["scale_dtype"]], self.cap, self.batch, int(S.QKV_BIAS), float(S.EPS),
                        float(S.ROPE_THETA), int(bool(cfg["keep_logits"])))
        self.tp, self.tp_rank = int(cfg.get("tp", 1)), int(cfg.get("tp_rank", 0))
        if self.tp > 1:
            if tp_id is None or len(tp_id) != 128:
                raise ValueError("DecodeModel: tensor parallelism needs the 128-byte communicator id (tp.exchange_id)")
            d.tp_world, d.tp_rank = self.tp, self.tp_rank
            C.memmove(d.tp_id, bytes(tp_id), 128)
        h = C.c_void_p()
        torch.cuda.set_device(device)
        N.check(N.lib().agxc_model_create(N.context(device), C.byref(d), C.byref(h)), "model_create")
        self._h = h
        off, cnt = C.c_int32(), C.c_int32()
        N.check(N.lib().agxc_model_vocab_slice(h, C.byref(off), C.byref(cnt)), "vocab_slice")
        self.vocab_offset, self.vocab_count = off.value, cnt.value
        self.packs = None   # reference-format packs kept on the host when build(keep_packs=True)

    @property
    def handle(self):
        return self._h

    # ---------------------------------------------------------------- weights
    def set_pack(self, layer, role, packed, scales, biases):
        """A reference-format pack (torch device tensors or numpy host arrays)."""
        on_dev = not isinstance(packed, np.ndarray)
        if on_dev:
            import torch
            torch.cuda.synchronize()
            args = [C.c_void_p(t.data_ptr()) for t in (packed, scales, biases)]
        else:
            arrs = [np.ascontiguousarray(a) for a in (packed, scales, biases)]
            args = [a.ctypes.data_as(C.c_void_p) for a in arrs]
        N.check(N.lib().agxc_model_set_pack(self._h, layer, ROLE[role], *args, int(on_dev)), "set_pack %s" % role)

    def set_vector(self, layer, which, data):
        """fp16 vector: which in {"attn_gain", "ffn_gain", "qkv_bias", "final_gain", "embed", "q_norm", "k_norm"}
        (the last two: the layer's QK-norm gains [head_dim])."""
        idx = {"attn_gain": N.VEC_ATTN_GAIN, "ffn_gain": N.VEC_FFN_GAIN, "qkv_bias": N.VEC_QKV_BIAS,
               "final_gain": N.VEC_FINAL_GAIN, "embed": N.VEC_EMBED, "q_norm": N.VEC_Q_NORM,
               "k_norm": N.VEC_K_NORM}[which]
        if isinstance(data, np.ndarray):
            a = np.ascontiguousarray(data.astype(np.float16, copy=False))
            N.check(N.lib().agxc_model_set_vector(self._h, layer, idx, a.ctypes.data_as(C.c_void_p), a.nbytes, 0),
                    "set_vector %s" % which)
        else:
            import torch
            t = data.to(torch.float16).contiguous()
            torch.cuda.synchronize()
            N.check(N.lib().agxc_model_set_vector(self._h, layer, idx, C.c_void_p(t.data_ptr()),
                                                  t.numel() * 2, 1), "set_vector %s" % which)

    OPTIONS = ("pdl", "trace", "fused", "bulk", "wait_ms", "tp_fused", "qk_norm", "device_wait_us")

    def set_option(self, option, value):
        """Model options: "fused" (batch 1 on one device: 1 = the whole step as one persistent kernel whose layer
        phases wait only on the counters of the data they read, where it fits; 0 (default) = one kernel per
        projection and attention in one CUDA graph, which measures faster at the 1.8B shape); "pdl" (the per-kernel path: programmatic dependent launch between the step's kernels: 0 off,
        1 (default) successor let in after the dependency wait, 2 after the inputs are staged, 3 after the last weight
        chunk); "trace" (the per-kernel path records each launch's CTA entry / wait / exit times, read with trace();
        the fused step records per-CTA phase times, read with trace_fused()); "bulk" (per-kernel GEMV weights by
        plain bulk copies instead of TMA tensor boxes); "wait_ms" (tensor parallel: the host's bound on a decode call,
        past which the communicator is aborted and TimeoutError raised; default 60000); "tp_fused" (tensor parallel:
        1 = the o_proj/down GEMMs push their tiles to every rank over NVLink and the sum is fused with the residual,
        the default where available; 0 = NCCL all-reduce; every rank must set the same value); "qk_norm" (Qwen3:
        the per-head RMSNorm of q and k before RoPE, with the "q_norm" / "k_norm" gains; build() sets it for a
        QK_NORM shape); "device_wait_us" (the bound on every wait of the fused step and the tensor-parallel reduce,
        default 2,000,000 us: a wait past it leaves the step undone and the call raises TimeoutError)."""
        opts = {"pdl": N.OPT_PDL, "trace": N.OPT_TRACE, "fused": N.OPT_FUSED, "bulk": N.OPT_BULK,
                "wait_ms": N.OPT_WAIT_MS, "tp_fused": N.OPT_TP_FUSED, "qk_norm": N.OPT_QK_NORM,
                "device_wait_us": N.OPT_DEVICE_WAIT_US}
        if option not in opts:
            raise ValueError("unknown option %r (known: %s)" % (option, sorted(opts)))
        N.check(N.lib().agxc_model_set_option(self._h, opts[option], int(value)), "set_option")

    @property
    def fused(self):
        """True when decode steps run as the fused persistent kernel."""
        return bool(self.plan_info()["fused"]["on"])

    def _trace_fused_rows(self):
        rows = FUSED_TRACE_MARKS * self.shape.LAYERS + 2 + len(FUSED_PROFILE_REGIONS)
        ctas = 256
        buf = (C.c_uint64 * (rows * ctas))()
        ph, ct = C.c_int32(), C.c_int32()
        N.check(N.lib().agxc_model_trace_cta_read(self._h, buf, rows * ctas, C.byref(ph), C.byref(ct)),
                "trace_cta_read")
        return np.frombuffer(buf, np.uint64)[: ph.value * ct.value].reshape(ph.value, ct.value).copy()

    def trace_fused(self):
        """The fused step's per-CTA marks of the last traced step (ns of the global timer, 0 = not reached): an array
        [marks, CTAs]; per layer twenty-six marks (0 qkv dependency met, 1 qkv done, 2 attention dependency met,
        3 attention done, 4 o_proj dependency met, 5 o_proj done, 6 FFN dependency met, 7 FFN done; 8 qkv input
        normed, 9 qkv tiles done, 10 attention keys done, 11 attention partials merged, 12 FFN input normed,
        13 first gate/up batch done, 14 gate/up done, 15 first down chunk done; the producer: 16 first qkv chunk
        issued, 17 attention chunks begin, 18 first FFN chunk issued, 19 last FFN chunk issued; 20 / 21 the qkv
        batch's first chunk landed / consumer thread 0's share done, 22 / 23 the same for the first gate/up batch, 24
        the second gate/up batch's first chunk landed, 25 the first down chunk issued), then the head's two."""
        return self._trace_fused_rows()[: FUSED_TRACE_MARKS * self.shape.LAYERS + 2]

    def profile_fused(self):
        """The fused step's cycle profile of the last traced step: {region: per-CTA SM cycles of consumer thread 0}
        (FUSED_PROFILE_REGIONS; thread 0 passes every consumer barrier, so the regions partition the CTA's time)."""
        tr = self._trace_fused_rows()[FUSED_TRACE_MARKS * self.shape.LAYERS + 2:]
        return {name: tr[k].astype(np.float64) for k, name in enumerate(FUSED_PROFILE_REGIONS) if name}

    def trace(self):
        """The launch trace since tracing started or the last call, then reset: one dict per launch of the step (in
        step order) with its kind and the first / last CTA entry, dependency-wait and exit times in ns, relative to
        the step's first entry."""
        cap = 5 * self.shape.LAYERS + 1
        W = 12
        buf = (C.c_uint64 * (W * cap))()
        n = C.c_int32()
        N.check(N.lib().agxc_model_trace_read(self._h, buf, cap, C.byref(n)), "trace_read")
        kinds = ["qkv", "attn", "wo", "ffn", "down"] * self.shape.LAYERS + ["head"]
        t0 = min(buf[W * i] for i in range(n.value))
        out = []
        for i in range(n.value):
            w = [buf[W * i + j] for j in range(W)]
            rec = dict(kind=kinds[i], entry=(w[0] - t0, w[1] - t0), wait=(w[2] - t0, w[3] - t0),
                       exit=(w[4] - t0, w[5] - t0))
            if w[7]:  # GEMV phases
                rec["staged"] = (w[6] - t0, w[7] - t0)
                rec["looped"] = (w[8] - t0, w[9] - t0)
                rec["landed"] = (w[10] - t0, w[11] - t0)
            out.append(rec)
        return out

    def plan_info(self):
        """The launch plan of every kernel of the step (dict)."""
        buf = C.create_string_buffer(4096)
        N.check(N.lib().agxc_model_plan_info(self._h, buf, 4096), "plan_info")
        return json.loads(buf.value.decode())

    @property
    def weight_bytes(self):
        return int(N.lib().agxc_model_weight_bytes(self._h))

    @property
    def kernels_per_step(self):
        n = C.c_int32()
        N.check(N.lib().agxc_model_kernel_count(self._h, C.byref(n)))
        return n.value

    # ---------------------------------------------------------------- sequences
    def start(self, b, prompt):
        p = np.ascontiguousarray(np.asarray(prompt, np.int32))
        N.check(N.lib().agxc_model_start(self._h, b, p.ctypes.data_as(C.c_void_p), p.size), "start")

    def prefill(self, b, prompt):
        """Start sequence b with its prompt and run positions 0 .. len-2 as the prefill section (chunks of up to 256
        rows on the tensor-core GEMM with causal attention); the next decode step runs the last prompt token. Returns
        {gpu_ms, host_ms, launches}."""
        p = np.ascontiguousarray(np.asarray(prompt, np.int32))
        t = N.Timing()
        N.check(N.lib().agxc_model_prefill(self._h, b, p.ctypes.data_as(C.c_void_p), p.size, C.byref(t)), "prefill")
        return dict(gpu_ms=t.gpu_ms, host_ms=t.host_ms, launches=t.launches_per_step)

    def verify(self, draft, b=0, want_logits=False):
        """The speculative verify step (agxc_model_verify): the current token and the drafted tokens as rows at
        q0 .. q0 + len(draft); returns (emitted tokens — the accepted drafts and the model's choice after them, all
        committed to the sequence —, the rows' logits [len(draft) + 1, V] or None)."""
        d = np.ascontiguousarray(np.asarray(draft, np.int32))
        if d.size > 15:
            raise ValueError("verify: at most 15 drafted tokens")
        out = np.zeros(16, np.int32)
        n = C.c_int32()
        lg = np.zeros((d.size + 1, self.vocab_count), np.float32) if want_logits else None
        N.check(N.lib().agxc_model_verify(self._h, b, d.ctypes.data_as(C.c_void_p) if d.size else None, d.size,
                                          out.ctypes.data_as(C.c_void_p), C.byref(n),
                                          None if lg is None else lg.ctypes.data_as(C.c_void_p)), "verify")
        return [int(t) for t in out[: n.value]], lg

    def force(self, b, pos, tokens):
        t = np.ascontiguousarray(np.asarray(tokens, np.int32))
        N.check(N.lib().agxc_model_force(self._h, b, pos, t.ctypes.data_as(C.c_void_p), t.size), "force")

    def fill_history(self, b, n, seed=0):
        N.check(N.lib().agxc_model_fill_history(self._h, b, n, seed), "fill_history")

    def state(self, b):
        q0 = np.zeros(1, np.uint32)
        log = np.zeros(self.cap, np.uint32)
        N.check(N.lib().agxc_model_state(self._h, b, q0.ctypes.data_as(C.c_void_p), log.ctypes.data_as(C.c_void_p)))
        return int(q0[0]), log

    def save_state(self, b=0):
        """Sequence b's decode state as bytes: q0, the token log, a pending forced token, the next input row and every
        layer's K/V rows 0 .. q0-1 (agxc_model_state_save's image)."""
        n = int(N.lib().agxc_model_state_bytes(self._h, b))
        if n < 0:
            N.check(n, "state_bytes")
        buf = C.create_string_buffer(n)
        w = C.c_size_t()
        N.check(N.lib().agxc_model_state_save(self._h, b, buf, n, C.byref(w)), "state_save")
        return buf.raw[: w.value]

    def restore_state(self, image, b=0):
        """Replace sequence b's decode state with a save_state() image (same shapes; the cap must hold it)."""
        data = bytes(image)
        buf = C.create_string_buffer(data, len(data))
        N.check(N.lib().agxc_model_state_restore(self._h, b, buf, len(data)), "state_restore")

    def read_kv(self, layer, b, n):
        S = self.shape
        k = np.zeros((S.KV_HEADS, n, S.HEAD_DIM), np.uint16)
        v = np.zeros_like(k)
        N.check(N.lib().agxc_model_read_kv(self._h, layer, b, n, k.ctypes.data_as(C.c_void_p),
                                           v.ctypes.data_as(C.c_void_p)), "read_kv")
        return k.view(np.float16), v.view(np.float16)

    def decode(self, steps, forced=None, want_tokens=True, want_logits=False, sync_each=False):
        """Run `steps` steps. Returns (tokens [steps, batch] or None, logits [steps, batch, V] or None, timing dict).
        sync_each: 0 / False waits once at the end; 1 / True waits for every step before queueing the next; 2 keeps
        one step queued ahead and waits for the step before it (each step's tokens reach the host one step later)."""
        if int(sync_each) not in (0, 1, 2):
            raise ValueError("decode: sync_each 0, 1 or 2")
        B, V = self.batch, self.vocab_count   # the rank's vocabulary slice under tensor parallelism
        toks = np.zeros((steps, B), np.int32) if want_tokens else None
        lg = np.zeros((steps, B, V), np.float32) if want_logits else None
        fin = None
        if forced is not None:
            fin = np.ascontiguousarray(np.asarray(forced, np.int64).astype(np.uint32).view(np.int32).reshape(steps, B))
        t = N.Timing()
        N.check(N.lib().agxc_decode(self._h, steps, None if fin is None else fin.ctypes.data_as(C.c_void_p),
                                    None if toks is None else toks.ctypes.data_as(C.c_void_p),
                                    None if lg is None else lg.ctypes.data_as(C.c_void_p), int(sync_each),
                                    C.byref(t)), "decode")
        return toks, lg, dict(gpu_ms=t.gpu_ms, host_ms=t.host_ms, launches_per_step=t.launches_per_step)

    def close(self):
        h = getattr(self, "_h", None)
        lib = getattr(N, "_lib", None) if N is not None else None
        if h and lib is not None:
            lib.agxc_model_free(h)
        self._h = None

    def __del__(self):
        self.close()


def synthetic_pack(torch, N_, K, bits, scale_dtype, gen, std, device):
    """N(0, std) fp32 weights generated on the device, quantised on the device: reference-format (packed, s, b)."""
    W = torch.randn((N_, K), generator=gen, device="cuda:%d" % device, dtype=torch.float32) * std
    out = Q.quantize(W, bits=bits, scale_dtype=scale_dtype, device=device)[:3]
    del W
    return out


def build(config, device=0, weights=None, keep_packs=False):
    """Create the device model. `weights` (optional) = dict with reference-format packs {(layer, role): (packed,
    scales, biases)} (roles qkv, wo, gate, up, down; (None, "head")) and fp16 vectors {"embed", "final_gain",
    (layer, "attn_gain"), (layer, "ffn_gain"), (layer, "qkv_bias")}; missing entries are generated synthetically.
    keep_packs=True keeps a host copy of every pack and vector in model.packs (for the CPU oracle); an integer n keeps
    the packs of the first n layers only (and the head)."""
    import torch
    if isinstance(config, int) and not isinstance(config, bool):
        if _current is None:
            raise ValueError("build(bits): configure a model first")
        config = dict(_current, bits=config)
        config.pop("shape", None)
        config["model"] = _current["shape"]
    cfg = configure(config)
    S = cfg["shape"]
    world, rank = cfg["tp"], cfg["tp_rank"]
    tp_id = TP.exchange_id(world, rank) if world > 1 else None
    m = DecodeModel(cfg, device, tp_id=tp_id)
    if S.QK_NORM:
        m.set_option("qk_norm", 1)
    bits, sdt, seed = m.bits, cfg["scale_dtype"], cfg["seed"]
    weights = weights or {}
    kept = {} if keep_packs else None

    def host(t):
        return t.cpu().numpy() if hasattr(t, "cpu") else t

    keep_layers = S.LAYERS if keep_packs is True else int(keep_packs or 0)

    def keep_pack(key, p):
        if kept is not None and (key[0] is None or key[0] < keep_layers):
            a, s, b = (host(x) for x in p)
            kept[key] = (a.view(np.uint32), s.view(np.uint16), b.view(np.uint16))

    # embedding first: a tied head is its quantisation
    emb = weights.get("embed")
    if emb is None:
        emb = (torch.randn((S.VOCAB, S.D_MODEL), generator=_gen(torch, seed, "embed"), device="cuda:%d" % device)
               * cfg["embed_std"]).to(torch.float16)
    m.set_vector(0, "embed", emb)
    if kept is not None:
        kept["embed"] = host(emb).astype(np.float16)
    for l in range(S.LAYERS):
        for role, n, k in S.matrices():
            p = weights.get((l, role))
            if p is None:
                p = synthetic_pack(torch, n, k, bits, sdt, _gen(torch, seed, l, role), cfg["init_std"], device)
            m.set_pack(l, role, *TP.shard_pack(role, p, S, bits, world, rank))
            keep_pack((l, role), p)
        for vec in ("attn_gain", "ffn_gain"):
            v = weights.get((l, vec))
            if v is not None:
                m.set_vector(l, vec, v)
            if kept is not None:
                kept[(l, vec)] = np.asarray(host(v), np.float16) if v is not None else np.ones(S.D_MODEL, np.float16)
        if S.QK_NORM:
            for vec in ("q_norm", "k_norm"):
                v = weights.get((l, vec))
                if v is None:   # synthetic: 1 + N(0, 0.1^2), so the gains matter
                    v = (1.0 + 0.1 * torch.randn((S.HEAD_DIM,), generator=_gen(torch, seed, l, vec),
                                                 device="cuda:%d" % device)).to(torch.float16)
                m.set_vector(l, vec, v)
                if kept is not None:
                    kept[(l, vec)] = np.asarray(host(v), np.float16)
        if S.QKV_BIAS:
            v = weights.get((l, "qkv_bias"))
            if v is None:
                v = (torch.randn((S.QKV,), generator=_gen(torch, seed, l, "bias"), device="cuda:%d" % device)
                     * cfg["bias_std"]).to(torch.float16)
            m.set_vector(l, "qkv_bias", TP.shard_bias(v, S, world, rank))
            if kept is not None:
                kept[(l, "qkv_bias")] = host(v).astype(np.float16)
    p = weights.get((None, "head"))
    if p is None:
        if S.TIED:
            e32 = emb.to(torch.float32) if hasattr(emb, "to") else torch.from_numpy(np.asarray(emb, np.float32)).cuda()
            p = Q.quantize(e32, bits=bits, scale_dtype=sdt, device=device)[:3]
        else:
            p = synthetic_pack(torch, S.VOCAB, S.D_MODEL, bits, sdt, _gen(torch, seed, "head"), cfg["init_std"], device)
    m.set_pack(0, "head", *TP.shard_pack("head", p, S, bits, world, rank))
    keep_pack((None, "head"), p)
    fg = weights.get("final_gain")
    if fg is not None:
        m.set_vector(0, "final_gain", fg)
    if kept is not None:
        kept["final_gain"] = np.asarray(host(fg), np.float16) if fg is not None else np.ones(S.D_MODEL, np.float16)
    torch.cuda.synchronize()
    m.packs = kept
    if os.environ.get("AGXC_FUSED") == "1" and m.batch == 1 and m.tp == 1 and m.plan_info()["fused"]["fits"]:
        m.set_option("fused", 1)      # the fused persistent step, for comparison runs
    return m
