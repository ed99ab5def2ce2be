"""Generate tests/golden/minilm_ref.npz from the reference's own complete-encoder reference.

Usage:  python tests/golden/make_minilm_golden.py <path of an AGXForge checkout>

Builds the reference's logical BERT graph (agxforge/g17/inferencegraph.py ``import_graph``, sentence pooling, 32
tokens) for the MiniLM-L6 shape over the seeded parameters of ``oracle.encoder.make_params(1)`` and runs the
reference's ``graph_reference`` (tools/g17inferencereference.py:18-99) under its two FP64 policies,
``original_fp64`` and ``half_transport_fp64``, on three 32-token inputs with padding masks of 32, 20 and 7 valid
tokens. Records the inputs, the sentence embeddings of both policies and, for the first case, the last layer's
hidden rows (fp64 policy). The checkout is only read; the npz is committed (the GPU box has no checkout).
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def main(ref_root):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ref_root, "tools"))
    sys.path.insert(0, ref_root)
    from agxforge.g17 import inferencegraph as IG
    import g17inferencereference as R
    from oracle import encoder as E

    params = E.make_params(1)
    specs, off = {}, 0
    for name, a in params.items():
        specs[name] = IG.Parameter(name, "F32", tuple(a.shape), off, off + a.nbytes)
        off += a.nbytes
    graph = IG.import_graph(dict(E.MINILM_L6), specs, tokens=32, sentence_pooling=True)
    rng = np.random.default_rng(20261202)
    out = {}
    for case, valid in enumerate((32, 20, 7)):
        ids = rng.integers(0, E.MINILM_L6["vocab_size"], 32).astype(np.int32)
        mask = np.array([1] * valid + [0] * (32 - valid), np.int32)
        inputs = dict(token_ids=ids, position_ids=np.arange(32, dtype=np.int32),
                      token_type_ids=np.zeros(32, np.int32), attention_mask=mask)
        out["case%d_token_ids" % case] = ids
        out["case%d_mask" % case] = mask
        for policy in ("original_fp64", "half_transport_fp64"):
            res = R.graph_reference(graph, params, inputs, policy=policy)
            out["case%d_%s_embedding" % (case, policy)] = res["sentence.embedding"]
            if case == 0 and policy == "original_fp64":
                out["case0_original_fp64_last_hidden"] = res["layer.5.ffn_norm"]
    np.savez_compressed(os.path.join(HERE, "minilm_ref.npz"), **out)
    print("wrote minilm_ref.npz:", sorted(out))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_minilm_golden.py <reference checkout>")
    main(sys.argv[1])
