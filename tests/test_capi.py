"""CPU checks of the C-ABI library: it loads, exports every function that
include/ltxq.h declares, and rejects bad arguments before touching a GPU."""

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = []
    for fn in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if fn.endswith(".h"):
            text = open(os.path.join(ROOT, "include", fn)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names += re.findall(r"\b(ltxq_[a-z0-9_]+)\s*\(", text)
    return sorted(set(names))


@pytest.fixture(scope="module")
def lib():
    from ltxq import _lib

    if not os.path.exists(_lib.LIB_PATH):
        import importlib.util

        spec = importlib.util.spec_from_file_location("ltxq_build", os.path.join(ROOT, "ltx-2-mlx_b200", "build.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build()
    return _lib.load()


def test_every_declared_symbol_is_exported(lib):
    declared = _declared()
    assert len(declared) >= 14
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"


def test_python_binding_covers_the_header():
    from ltxq import _lib

    assert set(_declared()) == set(_lib.SIGNATURES)


def test_version_and_error_text(lib):
    assert b"sm_100a" in lib.ltxq_version()


def test_argument_validation_without_gpu(lib):
    from ltxq import _lib

    st = lib.ltxq_qlinear(None, 4, None, None, None, None, 0, None)
    assert st == _lib.ERR_INVALID
    assert b"NULL" in lib.ltxq_last_error()
    q = _lib.QWeight(None, None, None, None, 64, 64, _lib.AFFINE, 3, 64, 0)
    st = lib.ltxq_dequantize(ctypes.byref(q), None, None)
    assert st == _lib.ERR_INVALID
    q = _lib.QWeight(1, 1, 1, None, 64, 64, _lib.AFFINE, 3, 64, 0)
    st = lib.ltxq_dequantize(ctypes.byref(q), 16, None)
    assert st == _lib.ERR_UNSUPPORTED
    pro = _lib.Prologue(_lib.NORM_RMS, 1e-6, _lib.Vec(16, _lib.F32, 0, 0, 0), _lib.Vec(16, _lib.F32, 0, 0, 0))
    st = lib.ltxq_adaln_modulate(16, _lib.BF16, 4, 12, ctypes.byref(pro), 16, None)
    assert st == _lib.ERR_UNSUPPORTED  # C % 8 != 0
