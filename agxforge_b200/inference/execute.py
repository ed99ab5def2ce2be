"""Running the decode loop and reporting it (the reference's agxforge/inference/execute.py:37-49 and its executor's
report, tools/g17decodegen.m:479-483,612-631).

    decode(model, tokens, out=None, pipelined=True, forced=None, timeout=900)

runs `tokens` decode steps of a built DecodeModel (agxforge_b200.inference.assemble.build) in-process through the C
ABI and returns the report dict with the reference's keys: out_ids (per sequence for a batch), tokens_per_s,
per_token_ms, gpu_ms_per_token, host_ms_per_token, dispatches_per_token, batch. `pipelined=True` launches every step's
graph back to back and reads the tokens once at the end (the reference's DECODEGEN_PIPELINED); False waits for each
step. `out` (optional path) receives the report as JSON, as the reference's executor writes it. A step that exceeds a
bounded device wait raises TimeoutError; other failures raise RuntimeError with the library's message.
"""
from __future__ import annotations

import json


def decode(model, tokens, out=None, pipelined=True, forced=None, timeout=900):
    steps = int(tokens)
    if steps < 0:
        raise ValueError("decode: tokens must be non-negative")
    toks, _, t = model.decode(steps, forced=forced, want_tokens=True, sync_each=not pipelined)
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
