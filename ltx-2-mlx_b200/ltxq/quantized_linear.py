"""Quantized linear layers over the reference's MLX cache layout.

``QuantizedLinear`` mirrors MLX ``nn.QuantizedLinear`` as the reference uses
it (LTX_2_MLX/loader/transformer_cache.py:1436-1462 builds the empty module,
:1238-1267 fills ``weight``/``scales``/``biases`` from ``mx.quantize``,
``bias`` stays bf16): the same attribute names and dtypes, the same
``mode``/``group_size``/``bits`` semantics and defaults (:797-811), and
``__call__(x) -> y``.  ``pretransposed=True`` gives the reference's
``_PretransposedQuantizedLinear`` (:177-193) whose packed arrays were built
from ``W.T``.

The forward pass is one launch of the sm_100a quantized GEMM with the
block's epilogue fused (bias, GELU, gated residual); there is no CPU path.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from .kernels import MXActivation, _require_cuda, _stream, prologue, vec_arg

QUANT_DEFAULTS = {"affine": (64, 4), "mxfp8": (32, 8)}
_MODE = {"affine": _lib.AFFINE, "mxfp8": _lib.MXFP8}
# how the GEMM computes (include/ltxq.h LTXQ_COMPUTE_*): "dequant" (bf16
# tensor cores over the exactly dequantized weight), "mx2" / "mx1" (native
# block-scaled fp8 MMAs on mxfp8 weights, activations in two / one MXFP8 terms)
COMPUTE = {"dequant": _lib.COMPUTE_DEQUANT, "mx2": _lib.COMPUTE_MX2, "mx1": _lib.COMPUTE_MX1}


def quant_defaults(mode: str, group_size: int | None, bits: int | None) -> tuple[int, int]:
    """``_quant_defaults`` (transformer_cache.py:797-811) for the modes this
    path implements."""
    if mode not in QUANT_DEFAULTS:
        raise ValueError(f"Unsupported quantization mode: {mode}")
    gs, b = QUANT_DEFAULTS[mode]
    return group_size or gs, bits or b


class QuantizedLinear:
    def __init__(self, weight: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor | None = None,
                 bias: torch.Tensor | None = None, *, group_size: int, bits: int, mode: str = "affine",
                 pretransposed: bool = False, in_features: int | None = None, out_features: int | None = None):
        if mode not in _MODE:
            raise ValueError(f"Unsupported quantization mode: {mode}")
        for t, name in ((weight, "weight"), (scales, "scales")):
            _require_cuda(t, name)
        self.weight = weight.contiguous()
        self.scales = scales.contiguous()
        self.biases = biases.contiguous() if biases is not None else None
        self.bias = bias.contiguous() if bias is not None else None
        self.group_size = int(group_size)
        self.bits = int(bits)
        self.mode = mode
        self.pretransposed = bool(pretransposed)
        packed_rows = self.weight.shape[0]
        packed_len = self.weight.shape[1] * 32 // self.bits
        if pretransposed:
            self.in_features = in_features or packed_rows
            self.out_features = out_features or packed_len
        else:
            self.out_features = out_features or packed_rows
            self.in_features = in_features or packed_len
        if mode == "affine" and self.biases is None:
            raise ValueError("affine quantization needs biases")
        self.compute = "dequant"

    def set_compute(self, compute: str) -> "QuantizedLinear":
        """Select how GEMMs over this weight compute (``COMPUTE``); the MX
        modes apply to mxfp8 weights in the standard layout, other weights
        keep the dequantizing kernels."""
        if compute not in COMPUTE:
            raise ValueError(f"unknown compute mode {compute!r}")
        self.compute = compute
        self._mx_scales = None
        if compute != "dequant":
            self.mx_scales()  # packed now, not inside a later stream capture
        return self

    def mx_scales(self) -> torch.Tensor | None:
        """The weight scales repacked for the MX modes' block-scaled MMA
        (``ltxq_mx_pack_weight_scales``), made once and again only when the
        scale tensor changes; None where the MX modes do not apply."""
        if getattr(self, "compute", "dequant") == "dequant" or self.mode != "mxfp8" or self.pretransposed:
            return None
        if self.in_features % 512 != 0:
            return None
        key = (self.scales.data_ptr(), self.scales._version)
        cached = getattr(self, "_mx_scales", None)
        if cached is None or cached[0] != key:
            lib = _lib.load()
            q = self._qweight_base(0, None)
            nbytes = lib.ltxq_mx_weight_scales_size(ctypes.byref(q))
            buf = torch.empty(nbytes, dtype=torch.uint8, device=self.scales.device)
            _lib.check(lib.ltxq_mx_pack_weight_scales(ctypes.byref(q), buf.data_ptr(), _stream()), "mx_pack_weight_scales")
            cached = (key, buf)
            self._mx_scales = cached
        return cached[1]

    # ------------------------------------------------------------------ build
    @classmethod
    def from_linear(cls, weight: torch.Tensor, bias: torch.Tensor | None = None, group_size: int | None = None,
                    bits: int | None = None, mode: str = "affine", pretransposed: bool = False) -> "QuantizedLinear":
        """Quantize a bf16 ``nn.Linear`` weight [out, in] on the GPU
        (``nn.QuantizedLinear.from_linear`` / ``mx.quantize``)."""
        _require_cuda(weight, "weight")
        gs, b = quant_defaults(mode, group_size, bits)
        w = weight.to(torch.bfloat16)
        n_out, k_in = w.shape
        src = w.t().contiguous() if pretransposed else w.contiguous()
        rows, length = src.shape
        packed = torch.empty((rows, length * b // 32), dtype=torch.uint32, device=w.device)
        if mode == "affine":
            scales = torch.empty((rows, length // gs), dtype=torch.bfloat16, device=w.device)
            biases = torch.empty_like(scales)
        else:
            scales = torch.empty((rows, length // gs), dtype=torch.uint8, device=w.device)
            biases = None
        q = _lib.QWeight(packed.data_ptr(), scales.data_ptr(), biases.data_ptr() if biases is not None else None,
                         None, n_out, k_in, _MODE[mode], b, gs,
                         _lib.LAYOUT_PRETRANSPOSED if pretransposed else _lib.LAYOUT_STD)
        _lib.check(_lib.load().ltxq_quantize(src.data_ptr(), ctypes.byref(q), _stream()), "quantize")
        bias_bf16 = bias.to(torch.bfloat16).contiguous() if bias is not None else None
        return cls(packed, scales, biases, bias_bf16, group_size=gs, bits=b, mode=mode,
                   pretransposed=pretransposed, in_features=k_in, out_features=n_out)

    # ------------------------------------------------------------------ views
    def _qweight_base(self, flags: int, mx_scales) -> _lib.QWeight:
        return _lib.QWeight(
            self.weight.data_ptr(), self.scales.data_ptr(),
            self.biases.data_ptr() if self.biases is not None else None,
            self.bias.data_ptr() if self.bias is not None else None,
            self.out_features, self.in_features, _MODE[self.mode], self.bits, self.group_size,
            _lib.LAYOUT_PRETRANSPOSED if self.pretransposed else _lib.LAYOUT_STD, flags,
            COMPUTE[getattr(self, "compute", "dequant")], mx_scales)

    def qweight(self) -> _lib.QWeight:
        mx = self.mx_scales()
        return self._qweight_base(self.data_flags(), mx.data_ptr() if mx is not None else None)

    def data_flags(self) -> int:
        """LTXQ_QW_* flags of the packed data (``ltxq_qweight_scan``), cached
        until the weight or scale tensors change (torch's in-place version
        counters).  ``fast_path = False`` asserts none (the general
        conversion everywhere)."""
        if self.mode != "mxfp8" or not getattr(self, "fast_path", True):
            return 0
        key = (self.weight.data_ptr(), self.weight._version, self.scales.data_ptr(), self.scales._version)
        cached = getattr(self, "_flags_cache", None)
        if cached is None or cached[0] != key:
            q = _lib.QWeight(self.weight.data_ptr(), self.scales.data_ptr(), None, None, self.out_features,
                             self.in_features, _MODE[self.mode], self.bits, self.group_size,
                             _lib.LAYOUT_PRETRANSPOSED if self.pretransposed else _lib.LAYOUT_STD, 0)
            flags = ctypes.c_uint32(0)
            _lib.check(_lib.load().ltxq_qweight_scan(ctypes.byref(q), ctypes.byref(flags), _stream()), "qweight_scan")
            cached = (key, int(flags.value))
            self._flags_cache = cached
        return cached[1]

    def dequantize(self) -> torch.Tensor:
        """bf16 weight: [out, in] (standard) or [in, out] (pretransposed)."""
        shape = (self.in_features, self.out_features) if self.pretransposed else (self.out_features, self.in_features)
        out = torch.empty(shape, dtype=torch.bfloat16, device=self.weight.device)
        q = self.qweight()
        _lib.check(_lib.load().ltxq_dequantize(ctypes.byref(q), out.data_ptr(), _stream()), "dequantize")
        return out

    def mx_terms(self, M: int) -> int:
        """Terms of the MX input a GEMM of M rows over this weight takes (2 for
        "mx2", 1 for "mx1"), or 0 where it runs the dequantizing kernels."""
        if self.compute == "dequant" or M <= 0:
            return 0
        q = self.qweight()
        if not _lib.load().ltxq_qlinear_mx_supported(M, ctypes.byref(q)):
            return 0
        return 2 if self.compute == "mx2" else 1

    # ---------------------------------------------------------------- forward
    def _epilogue(self, x_rows_shape, keep, gelu=False, residual=None, gate=None, gate_then_add=False):
        epi = _lib.Epilogue()
        if residual is not None:
            if gate is None:
                raise ValueError("gated epilogue needs a gate")
            _require_cuda(residual, "residual")
            if residual.dtype != torch.bfloat16:
                raise ValueError("residual must be bfloat16")
            residual = residual.contiguous()
            keep.append(residual)
            if residual.numel() != math.prod(x_rows_shape) * self.out_features:
                raise ValueError("residual shape does not match the output")
            epi.kind = _lib.EPI_GATE_THEN_ADD if gate_then_add else _lib.EPI_GATED_RESIDUAL
            epi.gate = vec_arg(gate, x_rows_shape, self.out_features, "gate", keep)
            epi.residual = residual.data_ptr()
        else:
            epi.kind = _lib.EPI_GELU if gelu else _lib.EPI_NONE
        return epi

    def __call__(self, x: torch.Tensor, *, gelu: bool = False, residual: torch.Tensor | None = None,
                 gate: torch.Tensor | None = None, gate_then_add: bool = False,
                 adaln: tuple | None = None, split_k: bool = True, mx_out: int = 0):
        """``y = x @ dequant(W).T + bias`` with optional fused consumers:
        ``gelu=True`` (project_in), ``residual``/``gate`` (gated residual add),
        and ``adaln=(scale, shift, eps[, norm])`` (the AdaLN prologue).

        ``split_k=False`` gives the library no workspace for split-K partials,
        so a GEMM with few tokens runs unsplit (one pass over K per tile).

        ``x`` may be an ``MXActivation`` (``mx_terms(M)`` terms): the
        block-scaled GEMM reads it directly (``ltxq_qlinear_mx``).  With such
        an input, ``mx_out`` 1 or 2 returns the result (bias, GELU applied) as
        an ``MXActivation`` of that many terms for the next GEMM."""
        if isinstance(x, MXActivation):
            return self._call_mx(x, gelu, residual, gate, gate_then_add, mx_out)
        if mx_out:
            raise ValueError("mx_out needs an MXActivation input (the block-scaled kernels)")
        _require_cuda(x, "x")
        if x.dtype != torch.bfloat16:
            raise ValueError(f"x must be bfloat16, got {x.dtype}")
        if x.shape[-1] != self.in_features:
            raise ValueError(f"x last dim {x.shape[-1]} != in_features {self.in_features}")
        x = x.contiguous()
        rows_shape = tuple(x.shape[:-1])
        M = x.numel() // self.in_features
        keep: list = []
        epi = self._epilogue(rows_shape, keep, gelu, residual, gate, gate_then_add)
        out = torch.empty(rows_shape + (self.out_features,), dtype=torch.bfloat16, device=x.device)
        q = self.qweight()
        lib = _lib.load()
        if adaln is not None:
            scale, shift, eps = adaln[:3]
            norm = adaln[3] if len(adaln) > 3 else "rms"
            nk = {"rms": _lib.NORM_RMS, "layer": _lib.NORM_LAYER, "none": _lib.NORM_NONE}[norm]
            pro = prologue(nk, eps, scale, shift, rows_shape, self.in_features, keep)
            ws_bytes = lib.ltxq_adaln_qlinear_workspace_size(M, ctypes.byref(q))
            ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device)
            _lib.check(lib.ltxq_adaln_qlinear(x.data_ptr(), M, ctypes.byref(pro), ctypes.byref(q), ctypes.byref(epi),
                                              out.data_ptr(), ws.data_ptr(), ws_bytes, _stream()), "adaln_qlinear")
        else:
            ws_bytes = lib.ltxq_qlinear_workspace_size(M, ctypes.byref(q)) if split_k else 0
            ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device) if ws_bytes else None
            _lib.check(lib.ltxq_qlinear(x.data_ptr(), M, ctypes.byref(q), ctypes.byref(epi), out.data_ptr(),
                                        ws.data_ptr() if ws is not None else None, ws_bytes, _stream()), "qlinear")
        return out

    def _call_mx(self, x: MXActivation, gelu, residual, gate, gate_then_add, mx_out):
        if x.K != self.in_features:
            raise ValueError(f"x last dim {x.K} != in_features {self.in_features}")
        if mx_out and residual is not None:
            raise ValueError("mx_out takes the none / GELU epilogues only")
        keep: list = []
        epi = self._epilogue(x.rows_shape, keep, gelu, residual, gate, gate_then_add)
        q = self.qweight()
        xs = x.struct()
        out = None
        out_struct = None
        if mx_out:
            out = MXActivation(x.rows_shape, self.out_features, mx_out, x.device)
            out_struct = out.struct()
            out_ptr = None
        else:
            out = torch.empty(x.rows_shape + (self.out_features,), dtype=torch.bfloat16, device=x.device)
            out_ptr = out.data_ptr()
        _lib.check(_lib.load().ltxq_qlinear_mx(ctypes.byref(xs), x.M, ctypes.byref(q), ctypes.byref(epi), out_ptr,
                                               ctypes.byref(out_struct) if out_struct is not None else None,
                                               _stream()), "qlinear_mx")
        return out

    def __repr__(self) -> str:
        return (f"QuantizedLinear(in={self.in_features}, out={self.out_features}, mode={self.mode}, "
                f"bits={self.bits}, group_size={self.group_size}, pretransposed={self.pretransposed})")
