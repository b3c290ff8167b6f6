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


def test_mx_entry_validation_without_gpu(lib):
    """The MX-form entry points reject bad activations / shapes before any
    CUDA call."""
    from ltxq import _lib

    q = _lib.QWeight(16, 16, None, None, 4096, 4096, _lib.MXFP8, 8, 32, 0, 0, _lib.COMPUTE_MX2, 16)
    epi = _lib.Epilogue()
    assert lib.ltxq_qlinear_mx(None, 256, ctypes.byref(q), ctypes.byref(epi), 16, None, None) == _lib.ERR_INVALID
    bad = _lib.MxAct(16, 16, 16, 16, 3, 0)  # three terms
    assert lib.ltxq_qlinear_mx(ctypes.byref(bad), 256, ctypes.byref(q), ctypes.byref(epi), 16, None,
                               None) == _lib.ERR_INVALID
    odd = _lib.MxAct(24, 16, 16, 16, 2, 0)  # codes not 16-byte aligned
    assert lib.ltxq_qlinear_mx(ctypes.byref(odd), 256, ctypes.byref(q), ctypes.byref(epi), 16, None,
                               None) == _lib.ERR_INVALID
    act = _lib.MxAct(16, 16, 16, 16, 2, 0)
    pro = _lib.Prologue(_lib.NORM_RMS, 1e-6, _lib.Vec(16, _lib.F32, 0, 0, 0), _lib.Vec(16, _lib.F32, 0, 0, 0))
    assert lib.ltxq_adaln_modulate_mx(16, 4, 4096, ctypes.byref(pro), None, None, None) == _lib.ERR_INVALID
    assert lib.ltxq_adaln_modulate_mx(16, 4, 4160, ctypes.byref(pro), None, ctypes.byref(act),
                                      None) == _lib.ERR_UNSUPPORTED  # C % 128 != 0
    assert lib.ltxq_adaln_modulate_mx(16, 4, 8192, ctypes.byref(pro), None, ctypes.byref(act),
                                      None) == _lib.ERR_UNSUPPORTED  # C > 4096
    assert lib.ltxq_head_gate_mx(16, 16, 4, 3, 64, None, ctypes.byref(act), None) == _lib.ERR_UNSUPPORTED
    assert lib.ltxq_head_gate_mx(16, 16, 4, 2, 64, None, None, None) == _lib.ERR_INVALID
    assert lib.ltxq_head_gate_ex(16, 16, 1, 4, 2, 64, 16, None, None) == _lib.ERR_INVALID  # stride < heads
    assert lib.ltxq_head_gate_ex(16, 16, 0, 4, 2, 64, 16, None, None) == _lib.ERR_INVALID  # stride not positive
    assert lib.ltxq_head_gate_ex(16, 16, 2, 0, 2, 64, 16, None, None) == _lib.OK            # no rows: no-op


def test_attention_validation_without_gpu(lib):
    """ltxq_attention rejects bad shapes / strides / pointers before any CUDA
    call, and an empty batch is a no-op."""
    from ltxq import _lib

    def call(q=16, k=16, v=16, b=1, tq=8, tk=8, h=2, d=64, qs=128, ks=128, vs=128, scale=0.125, out=16):
        return lib.ltxq_attention(q, k, v, b, tq, tk, h, d, qs, ks, vs, scale, out, None)

    assert call(q=None) == _lib.ERR_INVALID
    assert call(d=96, qs=192, ks=192, vs=192) == _lib.ERR_UNSUPPORTED  # head_dim
    assert call(tk=0) == _lib.ERR_INVALID
    assert call(qs=64) == _lib.ERR_INVALID                               # stride < heads * head_dim
    assert call(vs=132) == _lib.ERR_UNSUPPORTED                          # stride not a multiple of 8
    assert call(out=24) == _lib.ERR_UNSUPPORTED                          # 16-byte alignment
    assert call(scale=0.0) == _lib.ERR_INVALID
    assert call(b=0) == _lib.OK


def test_mx_activation_layout_on_cpu():
    """MXActivation: one buffer holding both terms' codes and scale atoms at
    256-byte aligned offsets, sized by ltxq_mx_split_sizes."""
    import torch

    from ltxq.kernels import MXActivation

    for M, K, terms in ((201, 2048, 2), (1000, 4096, 1), (1, 128, 2)):
        a = MXActivation((M,), K, terms, torch.device("cpu"))
        hi, lo, sf_hi, sf_lo = a.tensors()
        assert hi.shape == (M, K) and (lo is None) == (terms == 1)
        row_tiles = (M + 127) // 128 + 1
        assert sf_hi.numel() == (K // 128) * row_tiles * 512
        base = a.buffer.data_ptr()
        for p in a._parts:
            assert p is None or (p - base) % 256 == 0
        st = a.struct()
        assert st.terms == terms and st.hi == base


def test_denoise_update_validation_without_gpu(lib):
    """ltxq_denoise_update rejects bad scalars / shapes / missing operands
    before any CUDA call, and an empty latent is a no-op."""
    from ltxq import _lib

    def call(p, latent=16, v_cond=16, v_uncond=None, b=1, t=4, c=8, out=16, mask=None, clean=None, prev=None):
        return lib.ltxq_denoise_update(latent, v_cond, v_uncond, None, mask, clean, prev, b, t, c,
                                       None if p is None else ctypes.byref(p), out, None)

    ok = _lib.DenoiseParams(0.5, 0.25, 1.0, 0.0, 0.0, 0, 0)
    assert call(None) == _lib.ERR_INVALID
    assert call(_lib.DenoiseParams(0.0, 0.0, 1.0, 0.0, 0.0, 0, 0)) == _lib.ERR_INVALID  # sigma must be > 0
    assert b"sigma" in lib.ltxq_last_error()
    assert call(_lib.DenoiseParams(0.5, -0.1, 1.0, 0.0, 0.0, 0, 0)) == _lib.ERR_INVALID
    assert call(ok, c=12) == _lib.ERR_UNSUPPORTED  # channels % 8
    assert call(ok, latent=None) == _lib.ERR_INVALID
    assert call(_lib.DenoiseParams(0.5, 0.25, 3.0, 0.0, 0.0, 0, 0)) == _lib.ERR_INVALID  # CFG needs v_uncond
    assert call(_lib.DenoiseParams(0.5, 0.25, 1.0, 0.0, 1.5, 0, 0)) == _lib.ERR_INVALID  # ge needs prev_velocity
    assert call(ok, mask=16) == _lib.ERR_INVALID  # a mask needs the clean latent
    assert call(ok, latent=24) == _lib.ERR_UNSUPPORTED  # 16-byte alignment
    assert call(ok, latent=None, v_cond=None, out=None, b=0) == _lib.OK  # empty: nothing to do


def test_selftest_limits_checked_without_gpu(lib):
    from ltxq import _lib

    assert lib.ltxq_selftest_wait_timeout(0, None) == _lib.ERR_INVALID
    assert b"limit_ns" in lib.ltxq_last_error()
    assert lib.ltxq_selftest_wait_timeout(2_000_000_000, None) == _lib.ERR_INVALID
