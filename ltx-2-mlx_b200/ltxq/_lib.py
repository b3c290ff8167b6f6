"""ctypes binding of libltxq.so (the C ABI declared in include/ltxq.h).

The library is loaded from this package directory.  There is no fallback:
if the shared object is missing or cannot be loaded, every entry point
raises ``RuntimeError``.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int32, c_int64, c_size_t, c_void_p

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libltxq.so")

# status codes / enums (mirror include/ltxq.h)
OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA, ERR_DEVICE = 0, 1, 2, 3, 4
BF16, F32 = 0, 1
NORM_NONE, NORM_RMS, NORM_LAYER = 0, 1, 2
AFFINE, MXFP8 = 0, 1
LAYOUT_STD, LAYOUT_PRETRANSPOSED = 0, 1
QW_MXFP8_FINITE = 1
COMPUTE_DEQUANT, COMPUTE_MX2, COMPUTE_MX1 = 0, 1, 2
EPI_NONE, EPI_GELU, EPI_GATED_RESIDUAL, EPI_GATE_THEN_ADD = 0, 1, 2, 3
GATED_ADD, GATE_THEN_ADD = 0, 1


class QWeight(ctypes.Structure):
    _fields_ = [
        ("weight", c_void_p),
        ("scales", c_void_p),
        ("biases", c_void_p),
        ("bias", c_void_p),
        ("n_out", c_int64),
        ("k_in", c_int64),
        ("mode", c_int32),
        ("bits", c_int32),
        ("group_size", c_int32),
        ("layout", c_int32),
        ("flags", ctypes.c_uint32),
        ("compute", c_int32),
        ("mx_scales", c_void_p),
    ]


class Vec(ctypes.Structure):
    _fields_ = [
        ("ptr", c_void_p),
        ("dtype", c_int32),
        ("pad_", c_int32),
        ("rows_per_vec", c_int64),
        ("row_stride", c_int64),
    ]


class Epilogue(ctypes.Structure):
    _fields_ = [("kind", c_int32), ("pad_", c_int32), ("gate", Vec), ("residual", c_void_p)]


class Prologue(ctypes.Structure):
    _fields_ = [("norm", c_int32), ("eps", c_float), ("scale", Vec), ("shift", Vec)]


class MxAct(ctypes.Structure):
    _fields_ = [
        ("hi", c_void_p),
        ("lo", c_void_p),
        ("sf_hi", c_void_p),
        ("sf_lo", c_void_p),
        ("terms", c_int32),
        ("pad_", c_int32),
    ]


class DenoiseParams(ctypes.Structure):
    _fields_ = [
        ("sigma", c_float),
        ("sigma_next", c_float),
        ("cfg_scale", ctypes.c_double),
        ("stg_scale", ctypes.c_double),
        ("ge_gamma", ctypes.c_double),
        ("have_prev", c_int32),
        ("pad_", c_int32),
    ]


# name -> (restype, argtypes)
SIGNATURES = {
    "ltxq_last_error": (c_char_p, []),
    "ltxq_version": (c_char_p, []),
    "ltxq_device_error": (c_int32, [POINTER(c_int32)]),
    "ltxq_launch_count": (ctypes.c_uint64, []),
    "ltxq_selftest_wait_timeout": (c_int32, [ctypes.c_uint64, c_void_p]),
    "ltxq_qweight_scan": (c_int32, [POINTER(QWeight), POINTER(ctypes.c_uint32), c_void_p]),
    "ltxq_adaln_modulate": (c_int32, [c_void_p, c_int32, c_int64, c_int64, POINTER(Prologue), c_void_p, c_void_p]),
    "ltxq_gated_add": (c_int32, [c_void_p, c_void_p, POINTER(Vec), c_int64, c_int64, c_int32, c_void_p, c_void_p]),
    "ltxq_head_gate": (c_int32, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p]),
    "ltxq_qk_norm_rope": (c_int32, [c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p, c_float, c_void_p,
                                    c_void_p, c_int64, c_void_p, c_void_p]),
    "ltxq_qk_norm_rope_pair": (c_int32, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_void_p,
                                         c_void_p, c_float, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p]),
    "ltxq_attention": (c_int32, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64,
                                 c_int64, c_int64, c_float, c_void_p, c_void_p]),
    "ltxq_quantize": (c_int32, [c_void_p, POINTER(QWeight), c_void_p]),
    "ltxq_dequantize": (c_int32, [POINTER(QWeight), c_void_p, c_void_p]),
    "ltxq_qlinear_workspace_size": (c_size_t, [c_int64, POINTER(QWeight)]),
    "ltxq_adaln_qlinear_workspace_size": (c_size_t, [c_int64, POINTER(QWeight)]),
    "ltxq_feed_forward_workspace_size": (c_size_t, [c_int64, POINTER(QWeight), POINTER(QWeight)]),
    "ltxq_qlinear": (c_int32, [c_void_p, c_int64, POINTER(QWeight), POINTER(Epilogue), c_void_p, c_void_p,
                               c_size_t, c_void_p]),
    "ltxq_adaln_qlinear": (c_int32, [c_void_p, c_int64, POINTER(Prologue), POINTER(QWeight), POINTER(Epilogue),
                                     c_void_p, c_void_p, c_size_t, c_void_p]),
    "ltxq_mx_split_sizes": (c_size_t, [c_int64, c_int64, POINTER(c_size_t), POINTER(c_size_t)]),
    "ltxq_mx_weight_scales_size": (c_size_t, [POINTER(QWeight)]),
    "ltxq_mx_pack_weight_scales": (c_int32, [POINTER(QWeight), c_void_p, c_void_p]),
    "ltxq_mx_split": (c_int32, [c_void_p, c_int64, c_int64, c_int32, c_void_p, c_void_p, c_void_p, c_void_p,
                                c_void_p]),
    "ltxq_qlinear_mx_supported": (c_int32, [c_int64, POINTER(QWeight)]),
    "ltxq_qlinear_mx": (c_int32, [POINTER(MxAct), c_int64, POINTER(QWeight), POINTER(Epilogue), c_void_p,
                                  POINTER(MxAct), c_void_p]),
    "ltxq_adaln_modulate_mx": (c_int32, [c_void_p, c_int64, c_int64, POINTER(Prologue), c_void_p, POINTER(MxAct),
                                         c_void_p]),
    "ltxq_head_gate_mx": (c_int32, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, POINTER(MxAct),
                                    c_void_p]),
    "ltxq_head_gate_ex": (c_int32, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p,
                                    POINTER(MxAct), c_void_p]),
    "ltxq_adaln_qlinear_noalloc": (c_int32, [c_void_p, c_int64, POINTER(Prologue), POINTER(QWeight),
                                             POINTER(Epilogue), c_void_p, c_void_p]),
    "ltxq_feed_forward": (c_int32, [c_void_p, c_int64, POINTER(Prologue), POINTER(QWeight), POINTER(QWeight),
                                    POINTER(Epilogue), c_void_p, c_void_p, c_size_t, c_void_p]),
    "ltxq_denoise_update": (c_int32, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64,
                                      c_int64, c_int64, POINTER(DenoiseParams), c_void_p, c_void_p]),
}

_lib = None


class LtxqError(RuntimeError):
    pass


def load() -> ctypes.CDLL:
    """Load (once) and return the CUDA library; raise if it is unavailable."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"libltxq.so not found at {LIB_PATH}; build it with `python ltx-2-mlx_b200/build.py` "
            "(there is no CPU fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int, what: str = "") -> None:
    if status == OK:
        return
    msg = load().ltxq_last_error().decode(errors="replace")
    text = f"{what}: {msg}" if what else msg
    if status in (ERR_INVALID, ERR_UNSUPPORTED):
        raise ValueError(text)
    raise LtxqError(f"[status {status}] {text}")


def launch_count() -> int:
    """Kernels this library has launched in this process (host counter)."""
    return int(load().ltxq_launch_count())


def device_error() -> int:
    """Read and clear the device-side error word (synchronizes)."""
    code = c_int32(0)
    check(load().ltxq_device_error(ctypes.byref(code)), "device_error")
    return code.value
