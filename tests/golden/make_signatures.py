"""Record the reference's public signatures on the decode path (test infrastructure), so that the drop-in boundary
test can compare this package's functions with them without the reference checkout.

    python tests/golden/make_signatures.py <reference checkout>

writes tests/golden/ref_signatures.json: {"module.function": [parameter names with defaults]} for the functions of
agxforge.kernels.{qmv,attention,norm,argmax} and agxforge.inference.{catalog,assemble,execute} that the decode path's
callers use (the kernel-module and inference APIs of the path).
"""
import inspect
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))

NAMES = {
    "agxforge.kernels.qmv": ["quantize", "qmv_layout", "with_residual", "with_norm", "with_batch", "qmv_swiglu_layout",
                             "qmv2_ksplit_reference", "qmv2_reference_fast", "qmv_dq_reference",
                             "qmv_batch_reference", "qmv_swiglu_reference", "residual_reference"],
    "agxforge.kernels.attention": ["attn_layout", "attn_rope_layout", "attn_reference", "attn_rope_reference"],
    "agxforge.kernels.norm": ["rmsnorm_wide_reference"],
    "agxforge.kernels.argmax": ["argmax_reference"],
    "agxforge.inference.catalog": ["qmv_layout", "head_layout", "norm_layout", "attn_layout"],
    "agxforge.inference.assemble": ["configure", "build", "simulate"],
    "agxforge.inference.execute": ["decode", "executor"],
}


def describe(fn):
    out = []
    for p in inspect.signature(fn).parameters.values():
        d = None if p.default is inspect.Parameter.empty else repr(p.default)
        out.append([p.name, d])
    return out


def main(ref_root):
    sys.path.insert(0, ref_root)
    import importlib
    sigs = {}
    for mod, names in NAMES.items():
        m = importlib.import_module(mod)
        for n in names:
            sigs["%s.%s" % (mod, n)] = describe(getattr(m, n))
    with open(os.path.join(HERE, "ref_signatures.json"), "w") as f:
        json.dump(sigs, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_signatures.py <reference checkout>")
    main(sys.argv[1])
