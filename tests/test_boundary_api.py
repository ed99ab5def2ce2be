"""The drop-in boundary on the CPU: every reference function of the decode path that callers use exists here under
the reference's module path with the reference's parameters (names, order, defaults) as a prefix of ours, read from
tests/golden/ref_signatures.json (made by tests/golden/make_signatures.py from the reference checkout); the layout
records validate like the reference's (ValueError naming the constraint); and the ctypes stub INTEGRATION.md gives a
reference-side maintainer marshals a reference-format (bf16) pack and model descriptor correctly."""
import importlib
import inspect
import json
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

# where the B200 signature differs on purpose (the reason is in each function's docstring)
VARARGS = {"agxforge.inference.assemble.configure"}        # configure(config) or configure(deliver, config)
FIRST_ARG_RENAMED = {"agxforge.inference.assemble.build": "config"}   # build(bits) or build(config)


def _sigs():
    with open(os.path.join(ROOT, "tests", "golden", "ref_signatures.json")) as f:
        return json.load(f)


@pytest.mark.parametrize("name", sorted(_sigs()))
def test_reference_signature_is_a_prefix(name):
    ref = _sigs()[name]
    mod, fn = name.rsplit(".", 1)
    ours = getattr(importlib.import_module(mod), fn)
    params = list(inspect.signature(ours).parameters.values())
    if name in VARARGS:
        assert params[0].kind == inspect.Parameter.VAR_POSITIONAL
        return
    assert len(params) >= len(ref), (name, [p.name for p in params])
    for i, (rname, rdef) in enumerate(ref):
        p = params[i]
        want = FIRST_ARG_RENAMED.get(name) if i == 0 and name in FIRST_ARG_RENAMED else rname
        assert p.name == want, (name, i, p.name, rname)
        if rdef is not None:
            assert p.default is not inspect.Parameter.empty and repr(p.default) == rdef, (name, rname, p.default, rdef)
    for p in params[len(ref):]:
        assert p.default is not inspect.Parameter.empty or p.kind == inspect.Parameter.VAR_KEYWORD, (name, p.name)


def test_layouts_validate_like_the_reference():
    from agxforge.kernels import attention as A
    from agxforge.kernels import qmv as Q
    lay = Q.qmv_layout(4096, 2048, bits=4)
    assert lay["Nout"] == 4096 and lay["Kq"] == 2048 and lay["bits"] == 4
    with pytest.raises(ValueError, match="4- or 8-bit"):
        Q.qmv_layout(64, 256, bits=3)
    with pytest.raises(ValueError, match="group"):
        Q.qmv_layout(64, 100)
    with pytest.raises(ValueError, match="16"):
        Q.qmv_layout(40, 256, rows=4)
    with pytest.raises(ValueError):
        Q.with_residual(lay, "add8")
    assert Q.with_residual(lay, "add16")["res"] == "add16"
    sw = Q.qmv_swiglu_layout(8192, 2048)
    assert sw["swiglu"] and sw["ffn"] == 8192 and sw["Nout"] == 16384
    with pytest.raises(ValueError):
        A.attn_layout(head_dim=96)
    with pytest.raises(ValueError):
        A.attn_layout(heads=18, kv_heads=2)
    assert A.q_scale(128) == np.float32(1.4426950408889634 / np.sqrt(128))


def test_catalog_roles():
    from agxforge.inference import catalog, models
    for role in catalog.ROLES:
        lay, flags = catalog.qmv_layout(4, role, {"ks": 2})
        assert lay["bits"] == 4 and flags == ["ks"]
    with pytest.raises(ValueError):
        catalog.qmv_layout(4, "nope", None)
    lay, _ = catalog.head_layout(8, shape=models.QWEN25_05B)
    assert lay["Nout"] == 151936 and lay["tied"]
    assert catalog.attn_layout(2048)["cap"] == 2048


def test_configure_forms_and_simulate():
    from agxforge.inference import assemble
    a = assemble.configure({"model": "qwen2.5-0.5b", "bits": 8})
    b = assemble.configure("deliver-index-ignored", {"model": "qwen2.5-0.5b", "bits": 8})
    assert a["shape"] == b["shape"] and a["bits"] == b["bits"] == 8
    with pytest.raises(ValueError):
        assemble.configure({"bits": 5})
    with pytest.raises(NotImplementedError):
        assemble.simulate(4, 1)


def test_execute_decode_refuses_a_missing_library(tmp_path):
    from agxforge.inference import execute
    with pytest.raises(FileNotFoundError):
        execute.decode(object(), 1, None, binary=str(tmp_path / "missing.so"))


def _integration_stub():
    """The ctypes binding block INTEGRATION.md gives (the first ```python block after its stub heading)."""
    text = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    m = re.search(r"<!-- stub -->\s*```python\n(.*?)```", text, re.S)
    assert m, "INTEGRATION.md: the stub block is marked <!-- stub -->"
    return m.group(1)


def test_integration_stub_marshals_reference_packs():
    """Run the stub's marshalling (no library call): a reference-format pack from qmv.quantize carries bf16 scale and
    bias patterns, and the stub's model descriptor must say so (scale_dtype 1)."""
    ns = {}
    exec(compile(_integration_stub(), "INTEGRATION.md", "exec"), ns)
    rng = np.random.default_rng(0)
    from oracle import pack as P
    W = (rng.standard_normal((32, 128)) * 0.02).astype(np.float32)
    packed, s16, b16, q = P.quantize(W, bits=4, scale_dtype="bf16")     # the reference's own quantize format
    cfg = dict(d_model=2048, n_layers=24, n_heads=16, n_kv_heads=8, head_dim=128, ffn=8192, vocab=92544, bits=4,
               cap=2048, batch=1, eps=1e-5, rope_theta=1e6)
    desc = ns["model_desc"](cfg, scale_format="bf16")
    assert desc.scale_dtype == 1 and desc.bits == 4 and desc.group == 64
    assert ns["model_desc"](cfg, scale_format="fp16").scale_dtype == 0
    with pytest.raises(ValueError):
        ns["model_desc"](cfg, scale_format="fp32")
    args = ns["pack_args"](packed, s16, b16)
    assert [a.value for a in args] == [packed.ctypes.data, s16.ctypes.data, b16.ctypes.data]
    with pytest.raises(ValueError):
        ns["pack_args"](packed.astype(np.int64), s16, b16)
