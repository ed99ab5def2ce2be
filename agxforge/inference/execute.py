"""Running the decode loop and reporting it (the reference's agxforge/inference/execute.py:37-49 and its executor's
report, tools/g17decodegen.m:479-483,612-631).

    decode(graph, tokens, out, binary=None, pipelined=True, env=None, timeout=900)

The reference runs its Metal executor as a subprocess on a graph.json and reads back a JSON report. Here the executor
is in-process: `graph` is a built DecodeModel (assemble.build), or a config (dict or path of a JSON file) that is built
first. `tokens` decode steps run through the C ABI and the report carries the reference's keys: out_ids (per sequence
for a batch), tokens_per_s, per_token_ms, gpu_ms_per_token, host_ms_per_token, dispatches_per_token, batch. `out`
(a path, or None) receives the report as JSON, as the reference's executor writes it.

    binary      the native library (default: the in-tree libagxcuda.so); a path that is not a file raises
                FileNotFoundError, as the reference does for a missing executor (execute.py:40-41)
    pipelined   True (the reference's DECODEGEN_PIPELINED, its default): every step's graph is queued with one step in
                flight ahead of the host; False waits for each step before queueing the next
    env         switches, the reference's DECODEGEN_* environment: {"AGXC_PDL": "0"} and the like, one per model
                option (AGXC_<option>, see DecodeModel.set_option); None reads them from os.environ
    timeout     seconds; a run past it raises TimeoutError (a bounded device wait that gives up raises it too)

Failures raise RuntimeError with the library's message (the reference's stderr tail, execute.py:47-48).
"""
from __future__ import annotations

import json
import os

from agxforge_b200 import _native as N

OPTION_ENV = "AGXC_"


def executor():
    """The native library that runs the graph (the reference's executor binary, execute.py:32-34)."""
    return N.LIB_PATH


def _options(env):
    src = os.environ if env is None else env
    out = {}
    for k, v in src.items():
        if k.startswith(OPTION_ENV) and k != "AGXC_OPT_WAIT_MS" and len(k) > len(OPTION_ENV):
            out[k[len(OPTION_ENV):].lower()] = int(v)
    return out


def decode(graph, tokens, out=None, binary=None, pipelined=True, env=None, timeout=900, forced=None):
    if binary is not None and os.path.realpath(str(binary)) != os.path.realpath(N.LIB_PATH):
        if not os.path.isfile(str(binary)):
            raise FileNotFoundError("%s: build the library first (python -m agxforge_b200.build)" % binary)
        raise ValueError("decode: this package binds %s; another library is not loadable in the same process"
                         % N.LIB_PATH)
    if not os.path.isfile(N.LIB_PATH):
        raise FileNotFoundError("%s: build the library first (python -m agxforge_b200.build)" % N.LIB_PATH)
    steps = int(tokens)
    if steps < 0:
        raise ValueError("decode: tokens must be non-negative")
    model = graph
    if not hasattr(model, "decode"):
        from agxforge.inference import assemble
        model = assemble.build(graph)
    known = {"pdl", "trace", "bulk", "tp_fused", "fused"}
    for opt, val in _options(env).items():
        if opt in known:
            model.set_option(opt, val)
    model.set_option("wait_ms", int(min(timeout, 2 ** 31 // 1000 - 1) * 1000))
    toks, _, t = model.decode(steps, forced=forced, want_tokens=True, sync_each=2 if pipelined else 1)
    B = model.batch
    gpu_ms = t["gpu_ms"]
    host_ms = t["host_ms"]
    if host_ms / 1000.0 > timeout:
        raise TimeoutError("decode: %.1f s exceeded the %d s budget" % (host_ms / 1000.0, timeout))
    per_seq = [[int(v) for v in toks[:, b]] for b in range(B)]
    rep = dict(
        out_ids=per_seq[0] if B == 1 else per_seq,
        tokens_per_s=(steps * B) / (gpu_ms / 1000.0) if gpu_ms > 0 else 0.0,
        per_token_ms=gpu_ms / steps if steps else 0.0,
        gpu_ms_per_token=gpu_ms / steps if steps else 0.0,
        host_ms_per_token=host_ms / steps if steps else 0.0,
        dispatches_per_token=t["launches_per_step"],
        batch=B,
        pipelined=bool(pipelined),
    )
    if B > 1:
        rep["sequences"] = [dict(out_ids=s) for s in per_seq]
    if out is not None:
        with open(out, "w") as f:
            json.dump(rep, f, indent=1)
    return rep
