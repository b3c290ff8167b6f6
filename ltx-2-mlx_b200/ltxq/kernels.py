"""Drop-in replacements for ``LTX_2_MLX.kernels`` (fused_ops.py).

``adaln_norm_fused(x, scale, shift, eps)`` and ``gated_add_fused(residual,
branch, gate)`` keep the reference's names, argument order and return dtype
(fused_ops.py:237, 398).  Unlike the reference they never fall back to a
second implementation: every supported input (bf16/fp32 ``x``, fp32/bf16
vectors, broadcast, per-batch or per-token vectors, any eps, any C that is a
multiple of 8) runs the CUDA kernel, and anything else raises ``ValueError``.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _lib

_DT = {torch.bfloat16: _lib.BF16, torch.float32: _lib.F32}


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _require_cuda(t: torch.Tensor, name: str) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (there is no CPU path)")


def vec_arg(v: torch.Tensor, rows_shape: tuple[int, ...], C: int, name: str, keep: list) -> _lib.Vec:
    """Describe a per-channel vector broadcast against activations of shape
    ``rows_shape + (C,)``: all-singleton leading dims -> one vector for all
    rows; (B, 1, C) -> one vector per batch entry; (B, T, C) -> per token."""
    _require_cuda(v, name)
    if v.dtype not in _DT:
        raise ValueError(f"{name} dtype must be bfloat16 or float32, got {v.dtype}")
    if v.shape[-1] != C:
        raise ValueError(f"{name} last dim {v.shape[-1]} != {C}")
    if v.stride(-1) != 1:
        v = v.contiguous()
    keep.append(v)
    lead = tuple(v.shape[:-1])
    numel_lead = 1
    for d in lead:
        numel_lead *= d
    if numel_lead == 1:  # one vector for all rows (a strided view is used in place)
        return _lib.Vec(v.data_ptr(), _DT[v.dtype], 0, 0, 0)
    rows = 1
    for d in rows_shape:
        rows *= d
    if numel_lead == rows:  # (B, T, C): one vector per row
        if not v.is_contiguous():
            v = v.contiguous()
            keep.append(v)
        return _lib.Vec(v.data_ptr(), _DT[v.dtype], 0, 1, C)
    if len(rows_shape) >= 2 and len(lead) >= 1 and lead[0] == rows_shape[0] and numel_lead == rows_shape[0]:
        # (B, 1, C): one vector per batch entry, B vectors at the view's batch stride
        return _lib.Vec(v.data_ptr(), _DT[v.dtype], 0, rows // rows_shape[0], v.stride(0))
    raise ValueError(f"{name} shape {tuple(v.shape)} does not broadcast against {rows_shape + (C,)}")


class MXActivation:
    """Activations in the input form of the block-scaled GEMMs
    (``ltxq_mx_act``: per term [M, K] E4M3 codes and E8M0 scales in the MMA's
    atom layout; ``terms`` 2 or 1).  Written by ``adaln_modulate`` /
    ``head_gate`` with ``mx_terms`` and by ``QuantizedLinear`` with
    ``mx_out``, read by ``QuantizedLinear``; the bits are those
    ``ltxq_mx_split`` gives for the bf16 values.  One device buffer holds
    every part."""

    def __init__(self, rows_shape: tuple[int, ...], K: int, terms: int, device):
        if terms not in (1, 2):
            raise ValueError("terms must be 1 or 2")
        self.rows_shape = tuple(rows_shape)
        self.K = int(K)
        self.terms = int(terms)
        self.M = math.prod(self.rows_shape)
        codes, sf = ctypes.c_size_t(0), ctypes.c_size_t(0)
        if not _lib.load().ltxq_mx_split_sizes(self.M, self.K, ctypes.byref(codes), ctypes.byref(sf)):
            raise ValueError(f"no MX form for {self.M} x {self.K} (K % 128 == 0 and M > 0 needed)")
        cb, sb = _align(codes.value), _align(sf.value)
        self.buffer = torch.empty(terms * (cb + sb), dtype=torch.uint8, device=device)
        base = self.buffer.data_ptr()
        self._parts = (base, base + cb if terms == 2 else None, base + terms * cb,
                       base + terms * cb + sb if terms == 2 else None)

    @property
    def shape(self) -> tuple[int, ...]:
        return self.rows_shape + (self.K,)

    @property
    def device(self):
        return self.buffer.device

    def tensors(self) -> tuple:
        """(hi, lo, sf_hi, sf_lo) as uint8 views of the buffer: codes [M, K],
        scale atoms flat (ltxq_mx_split_sizes bytes); lo / sf_lo None for one
        term."""
        codes, sf = ctypes.c_size_t(0), ctypes.c_size_t(0)
        _lib.load().ltxq_mx_split_sizes(self.M, self.K, ctypes.byref(codes), ctypes.byref(sf))
        base = self.buffer.data_ptr()
        out = []
        for ptr, n, shape in zip(self._parts, (codes.value, codes.value, sf.value, sf.value),
                                 ((self.M, self.K), (self.M, self.K), (-1,), (-1,))):
            out.append(None if ptr is None else self.buffer[ptr - base:ptr - base + n].view(shape))
        return tuple(out)

    def struct(self) -> _lib.MxAct:
        hi, lo, sf_hi, sf_lo = self._parts
        return _lib.MxAct(hi, lo, sf_hi, sf_lo, self.terms, 0)

    @classmethod
    def split(cls, x: torch.Tensor, terms: int) -> "MXActivation":
        """The MX form of bf16 ``x`` (``ltxq_mx_split``)."""
        _require_cuda(x, "x")
        if x.dtype != torch.bfloat16:
            raise ValueError("x must be bfloat16")
        x = x.contiguous()
        act = cls(tuple(x.shape[:-1]), x.shape[-1], terms, x.device)
        hi, lo, sf_hi, sf_lo = act._parts
        _lib.check(_lib.load().ltxq_mx_split(x.data_ptr(), act.M, act.K, terms, hi, lo, sf_hi, sf_lo, _stream()),
                   "mx_split")
        return act


def _align(n: int) -> int:
    return (n + 255) & ~255


def mx_output_ok(C: int) -> bool:
    """Whether the row kernels (AdaLN, head gate) can write C channels in the
    MX form (32-channel groups held by lane quads, at most 4096 channels for
    the AdaLN pass)."""
    return C % 128 == 0 and C <= 4096


def prologue(norm: int, eps: float, scale, shift, rows_shape, C, keep) -> _lib.Prologue:
    return _lib.Prologue(norm, float(eps), vec_arg(scale, rows_shape, C, "scale", keep),
                         vec_arg(shift, rows_shape, C, "shift", keep))


def adaln_modulate(x: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor, eps: float = 1e-6,
                   norm: str = "rms", mx_terms: int = 0):
    """``bf16(norm(x) * (1 + scale) + shift)`` with norm in {"rms", "layer",
    "none"}; "none" is the text cross-attention context modulation
    (transformer.py:379).  ``mx_terms`` 1 or 2 returns the result as an
    ``MXActivation`` instead (the next block-scaled GEMM's input; bf16 x,
    ``mx_output_ok(C)``)."""
    _require_cuda(x, "x")
    if x.dtype not in _DT:
        raise ValueError(f"x dtype must be bfloat16 or float32, got {x.dtype}")
    x = x.contiguous()
    C = x.shape[-1]
    rows_shape = tuple(x.shape[:-1])
    keep: list = []
    nk = {"rms": _lib.NORM_RMS, "layer": _lib.NORM_LAYER, "none": _lib.NORM_NONE}[norm]
    pro = prologue(nk, eps, scale, shift, rows_shape, C, keep)
    lib = _lib.load()
    if mx_terms:
        act = MXActivation(rows_shape, C, mx_terms, x.device)
        st = act.struct()
        _lib.check(lib.ltxq_adaln_modulate_mx(x.data_ptr(), act.M, C, ctypes.byref(pro), None, ctypes.byref(st),
                                              _stream()), "adaln_modulate_mx")
        return act
    out = torch.empty_like(x)
    _lib.check(lib.ltxq_adaln_modulate(x.data_ptr(), _DT[x.dtype], x.numel() // C, C, ctypes.byref(pro),
                                       out.data_ptr(), _stream()), "adaln_modulate")
    return out


def adaln_norm_fused(x: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor, eps: float) -> torch.Tensor:
    """``(rms_norm(x) * (1 + scale) + shift).astype(x.dtype)``
    (fused_ops.py:237 / transformer.py:21-37)."""
    return adaln_modulate(x, scale, shift, eps, "rms")


def gated_add_fused(residual: torch.Tensor, branch: torch.Tensor, gate: torch.Tensor,
                    gate_then_add: bool = False) -> torch.Tensor:
    """``(residual + branch * gate).astype(residual.dtype)``
    (fused_ops.py:398 / transformer.py:40-50).  ``gate_then_add=True`` gives
    the text cross-attention form ``residual + bf16(branch * gate)``
    (transformer.py:387, 484)."""
    _require_cuda(residual, "residual")
    _require_cuda(branch, "branch")
    if residual.dtype != torch.bfloat16 or branch.dtype != torch.bfloat16:
        raise ValueError("residual and branch must be bfloat16")
    if residual.shape != branch.shape:
        raise ValueError(f"shape mismatch {tuple(residual.shape)} vs {tuple(branch.shape)}")
    residual = residual.contiguous()
    branch = branch.contiguous()
    C = residual.shape[-1]
    keep: list = []
    g = vec_arg(gate, tuple(residual.shape[:-1]), C, "gate", keep)
    out = torch.empty_like(residual)
    mode = _lib.GATE_THEN_ADD if gate_then_add else _lib.GATED_ADD
    _lib.check(_lib.load().ltxq_gated_add(residual.data_ptr(), branch.data_ptr(), ctypes.byref(g),
                                          residual.numel() // C, C, mode, out.data_ptr(), _stream()),
               "gated_add")
    return out


def head_gate(out: torch.Tensor, gate_logits: torch.Tensor, heads: int, mx_terms: int = 0):
    """``out * (2 * sigmoid(gate_logits))[..., None]`` per head
    (attention.py:559-601).  ``mx_terms`` as in ``adaln_modulate``.
    ``gate_logits`` may be a column slice of a wider tensor (rows at a
    uniform stride, heads contiguous): it is read in place."""
    _require_cuda(out, "out")
    _require_cuda(gate_logits, "gate_logits")
    if out.dtype != torch.bfloat16 or gate_logits.dtype != torch.bfloat16:
        raise ValueError("head_gate expects bfloat16 tensors")
    out = out.contiguous()
    width = out.shape[-1]
    rows = out.numel() // width
    if gate_logits.numel() != rows * heads or gate_logits.shape[-1] != heads:
        raise ValueError("gate_logits must have one value per (row, head)")
    try:
        gl = gate_logits.view(rows, heads)
    except RuntimeError:  # rows not at one uniform stride
        gl = gate_logits.contiguous().view(rows, heads)
    if gl.stride(1) != 1 or (rows > 1 and gl.stride(0) < heads):
        gl = gl.contiguous()
    lstride = gl.stride(0) if rows > 1 else heads
    if mx_terms:
        act = MXActivation(tuple(out.shape[:-1]), width, mx_terms, out.device)
        st = act.struct()
        _lib.check(_lib.load().ltxq_head_gate_ex(out.data_ptr(), gl.data_ptr(), lstride, rows, heads, width // heads,
                                                 None, ctypes.byref(st), _stream()), "head_gate_ex")
        return act
    res = torch.empty_like(out)
    _lib.check(_lib.load().ltxq_head_gate_ex(out.data_ptr(), gl.data_ptr(), lstride, rows, heads, width // heads,
                                             res.data_ptr(), None, _stream()), "head_gate_ex")
    return res


def qk_norm_rope_pair(q: torch.Tensor, k: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor, heads: int,
                      eps: float = 1e-6, pe: tuple | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """``qk_norm_rope`` of Q and K over the same rows and RoPE tables in one
    pass (the tables are read once): the self-attention's Q/K norm and
    rotation (attention.py:580-587)."""
    for t, name in ((q, "q"), (k, "k")):
        _require_cuda(t, name)
        if t.dtype != torch.bfloat16 or t.stride(-1) != 1 or t.dim() != 3:
            raise ValueError(f"{name} must be a (B, T, W) bfloat16 tensor with unit column stride")
    if q.shape != k.shape:
        raise ValueError("q and k must have the same shape")
    b, t, width = q.shape
    q = q if q.stride(0) == t * q.stride(1) else q.contiguous()
    k = k if k.stride(0) == t * k.stride(1) else k.contiguous()
    d = width // heads
    wq, wk = q_weight.float().contiguous(), k_weight.float().contiguous()
    oq = torch.empty((b, t, width), dtype=torch.bfloat16, device=q.device)
    ok = torch.empty_like(oq)
    cos = sin = None
    if pe is not None:
        cos, sin = pe[0].float().contiguous(), pe[1].float().contiguous()
        if cos.shape != (b, heads, t, d // 2) and cos.shape != (1, heads, t, d // 2):
            raise ValueError(f"RoPE table shape {tuple(cos.shape)} does not match {(b, heads, t, d // 2)}")
        if cos.shape[0] != b:
            cos, sin = cos.expand(b, -1, -1, -1).contiguous(), sin.expand(b, -1, -1, -1).contiguous()
    _lib.check(_lib.load().ltxq_qk_norm_rope_pair(
        q.data_ptr(), k.data_ptr(), b * t, q.stride(1), k.stride(1), heads, d, wq.data_ptr(), wk.data_ptr(),
        float(eps), cos.data_ptr() if cos is not None else None, sin.data_ptr() if sin is not None else None, t,
        oq.data_ptr(), ok.data_ptr(), _stream()), "qk_norm_rope_pair")
    return oq, ok


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, heads: int, scale: float | None = None) -> torch.Tensor:
    """``softmax(q k^T * scale) v`` per head (the block's
    ``mx.fast.scaled_dot_product_attention``, attention.py:170-302) on
    (B, T, heads*D) rows: q (B, Tq, W), k / v (B, Tk, W), any row stride with
    unit column stride (column slices of a fused projection are read in
    place).  D = W / heads must be 64 or 128; scale defaults to 1/sqrt(D).
    Returns contiguous (B, Tq, heads*D) bf16."""
    for t, name in ((q, "q"), (k, "k"), (v, "v")):
        _require_cuda(t, name)
        if t.dtype != torch.bfloat16 or t.dim() != 3 or t.stride(-1) != 1:
            raise ValueError(f"{name} must be a (B, T, W) bfloat16 tensor with unit column stride")
    b, tq, width = q.shape
    if k.shape != v.shape or k.shape[0] != b or k.shape[2] != width:
        raise ValueError("k and v must be (B, Tk, W) with q's B and W")
    tk = k.shape[1]
    if width % heads != 0:
        raise ValueError("W must be a multiple of heads")
    d = width // heads
    if scale is None:
        scale = 1.0 / math.sqrt(d)

    def rows(t):  # (B, T, W) with one row stride across batch and tokens
        if t.stride(0) != t.shape[1] * t.stride(1):
            t = t.contiguous()
        return t

    q, k, v = rows(q), rows(k), rows(v)
    out = torch.empty((b, tq, width), dtype=torch.bfloat16, device=q.device)
    _lib.check(_lib.load().ltxq_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), b, tq, tk, heads, d, q.stride(1),
                                          k.stride(1), v.stride(1), float(scale), out.data_ptr(), _stream()),
               "attention")
    return out


def qk_norm_rope(x: torch.Tensor, weight: torch.Tensor, heads: int, eps: float = 1e-6,
                 pe: tuple | None = None) -> torch.Tensor:
    """QK RMSNorm (attention.py:320-329) then split RoPE (rope.py:53-90) in one
    pass.  x: (B, T, heads*D) bf16, any row stride with unit column stride;
    pe: (cos, sin) fp32 (B, heads, T, D/2) or None.  Returns contiguous
    (B, T, heads*D) bf16."""
    _require_cuda(x, "x")
    if x.dtype != torch.bfloat16 or x.stride(-1) != 1 or x.dim() != 3:
        raise ValueError("x must be a (B, T, W) bfloat16 tensor with unit column stride")
    b, t, width = x.shape
    if x.stride(0) != t * x.stride(1):
        x = x.contiguous()
    d = width // heads
    w = weight.float().contiguous()
    out = torch.empty((b, t, width), dtype=torch.bfloat16, device=x.device)
    cos = sin = None
    if pe is not None:
        cos, sin = pe[0].float().contiguous(), pe[1].float().contiguous()
        if cos.shape != (b, heads, t, d // 2) and cos.shape != (1, heads, t, d // 2):
            raise ValueError(f"RoPE table shape {tuple(cos.shape)} does not match {(b, heads, t, d // 2)}")
        if cos.shape[0] != b:
            cos, sin = cos.expand(b, -1, -1, -1).contiguous(), sin.expand(b, -1, -1, -1).contiguous()
    _lib.check(_lib.load().ltxq_qk_norm_rope(x.data_ptr(), b * t, x.stride(1), heads, d, w.data_ptr(), float(eps),
                                             cos.data_ptr() if cos is not None else None,
                                             sin.data_ptr() if sin is not None else None, t, out.data_ptr(),
                                             _stream()), "qk_norm_rope")
    return out
