"""``FeedForward`` over quantized projections (feed_forward.py:39-112).

``FeedForward(project_in, project_out)`` computes
``project_out(gelu_approx(project_in(x)))`` like the reference's
``FeedForward.__call__`` (feed_forward.py:64-80, ``_project_in`` :101-102).
``sublayer`` is the whole FF sub-layer of the block (transformer.py:629-668):
AdaLN prologue, the two quantized GEMMs (GELU fused into the first one's
epilogue) and the gated residual fused into the second one's epilogue, as
one ``ltxq_feed_forward`` call.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .kernels import _require_cuda, _stream, prologue, vec_arg
from .quantized_linear import QuantizedLinear


class FeedForward:
    def __init__(self, project_in: QuantizedLinear, project_out: QuantizedLinear):
        if project_out.in_features != project_in.out_features:
            raise ValueError("project_out.in_features must equal project_in.out_features")
        self.project_in = project_in
        self.project_out = project_out
        self.dim = project_in.in_features
        self.inner_dim = project_in.out_features
        self.dim_out = project_out.out_features

    @classmethod
    def from_linear(cls, w_in, b_in, w_out, b_out, mode: str = "affine", group_size: int | None = None,
                    bits: int | None = None) -> "FeedForward":
        return cls(QuantizedLinear.from_linear(w_in, b_in, group_size, bits, mode),
                   QuantizedLinear.from_linear(w_out, b_out, group_size, bits, mode))

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return self._run(x, None, None)

    def sublayer(self, x: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor, gate: torch.Tensor,
                 eps: float = 1e-6, norm: str = "rms") -> torch.Tensor:
        """``x + gate * FF(modulate(norm(x)))`` (transformer.py:629-668)."""
        return self._run(x, (scale, shift, eps, norm), gate)

    def _run(self, x, adaln, gate):
        _require_cuda(x, "x")
        if x.dtype != torch.bfloat16:
            raise ValueError("x must be bfloat16")
        if x.shape[-1] != self.dim:
            raise ValueError(f"x last dim {x.shape[-1]} != {self.dim}")
        x = x.contiguous()
        rows_shape = tuple(x.shape[:-1])
        M = x.numel() // self.dim
        keep: list = []
        lib = _lib.load()
        qi, qo = self.project_in.qweight(), self.project_out.qweight()
        pro_p = None
        if adaln is not None:
            scale, shift, eps, norm = adaln
            nk = {"rms": _lib.NORM_RMS, "layer": _lib.NORM_LAYER, "none": _lib.NORM_NONE}[norm]
            pro = prologue(nk, eps, scale, shift, rows_shape, self.dim, keep)
            pro_p = ctypes.byref(pro)
        epi = _lib.Epilogue()
        if gate is not None:
            if self.dim_out != self.dim:
                raise ValueError("gated residual needs dim_out == dim")
            epi.kind = _lib.EPI_GATED_RESIDUAL
            epi.gate = vec_arg(gate, rows_shape, self.dim_out, "gate", keep)
            epi.residual = x.data_ptr()
        else:
            epi.kind = _lib.EPI_NONE
        out = torch.empty(rows_shape + (self.dim_out,), dtype=torch.bfloat16, device=x.device)
        ws_bytes = lib.ltxq_feed_forward_workspace_size(M, ctypes.byref(qi), ctypes.byref(qo))
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device)
        _lib.check(lib.ltxq_feed_forward(x.data_ptr(), M, pro_p, ctypes.byref(qi), ctypes.byref(qo), ctypes.byref(epi),
                                         out.data_ptr(), ws.data_ptr(), ws_bytes, _stream()), "feed_forward")
        return out
