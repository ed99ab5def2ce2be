"""The C-ABI library: it loads, exports every entry point include/agxc.h declares, and fails loudly without a GPU.
No compute calls here (no GPU in the CPU suite)."""
import ctypes
import os
import re

import pytest

from agxforge_b200 import _native as N

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "agxc.h")).read()
    return sorted(set(re.findall(r"^AGXC_API [^(]*?\b(agxc_\w+)\(", text, re.M)))


@pytest.fixture(scope="module")
def built():
    from agxforge_b200 import build
    return build.build()


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert len(syms) >= 25
    assert "agxc_decode" in syms and "agxc_qmv" in syms and "agxc_attention_dev" in syms


def test_library_exports_every_declared_symbol(built):
    lib = ctypes.CDLL(built)
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_binding_covers_header():
    # every declared entry point has a ctypes signature in the binding
    assert sorted(N.SIGNATURES) == declared_symbols()


def test_version_and_error_without_gpu(built):
    import torch
    L = N.lib()
    assert L.agxc_version() == 1
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    p = ctypes.c_void_p()
    rc = L.agxc_init(0, ctypes.byref(p))
    assert rc != 0
    assert L.agxc_last_error()


def test_context_raises_without_gpu(built):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    with pytest.raises((RuntimeError, ValueError)):
        N.context(0)


def test_product_fails_loudly_without_library(monkeypatch, tmp_path):
    monkeypatch.setattr(N, "_lib", None)
    monkeypatch.setattr(N, "LIB_PATH", str(tmp_path / "missing.so"))
    with pytest.raises(FileNotFoundError):
        N.lib()


@pytest.mark.parametrize("package", ["agxforge", "agxforge_b200"])
def test_package_never_imports_oracle(package):
    pkg = os.path.join(ROOT, package)
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h")):
                text = open(os.path.join(dirpath, f)).read()
                assert not re.search(r"^\s*(from|import)\s+oracle\b", text, re.M), f
