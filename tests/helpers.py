"""Shared test helpers: seeded inputs (numpy PCG64 -> fp32 -> bf16 RNE, the
generator the benchmark configs are drawn with) and numpy <-> torch moves."""

from __future__ import annotations

import numpy as np

from oracle.bf16 import bf16_bits_to_f32, f32_to_bf16_bits, rbf16


def rng(seed: int = 0) -> np.random.Generator:
    return np.random.default_rng(seed)


def normal_bf16(g: np.random.Generator, shape, std: float = 1.0) -> np.ndarray:
    return rbf16((g.standard_normal(shape) * std).astype(np.float32))


def normal_f32(g: np.random.Generator, shape, std: float = 1.0) -> np.ndarray:
    return (g.standard_normal(shape) * std).astype(np.float32)


def to_dev_bf16(a: np.ndarray, device="cuda"):
    import torch

    bits = f32_to_bf16_bits(np.asarray(a, dtype=np.float32))
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).to(device)


def to_dev(a: np.ndarray, device="cuda"):
    import torch

    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        return torch.from_numpy(a.view(np.int32).copy()).view(torch.uint32).to(device)
    if a.dtype == np.uint16:  # bf16 bit patterns
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16).to(device)
    return torch.from_numpy(a.copy()).to(device)


def from_dev_bf16(t) -> np.ndarray:
    import torch

    bits = t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    return bf16_bits_to_f32(bits)


def bf16_bits(t) -> np.ndarray:
    import torch

    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def ulp_diff_bf16(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """|a - b| in units of bf16 ulps (sign-magnitude ordering)."""
    ia = f32_to_bf16_bits(a).astype(np.int32)
    ib = f32_to_bf16_bits(b).astype(np.int32)
    ia = np.where(ia & 0x8000, 0x8000 - ia, ia)
    ib = np.where(ib & 0x8000, 0x8000 - ib, ib)
    return np.abs(ia - ib)


def block_params(video, audio, mode: str, bits: int, seed: int = 30):
    """One block's random parameters: (oracle params with dequantized bf16
    weights, {base: (packed numpy arrays, bias)}, fp32 tables)."""
    from ltxq.block import linear_specs, table_specs
    from oracle import quant as oq

    g = rng(seed)
    p_oracle, quant = {}, {}
    for name, (n, k) in linear_specs(video, audio).items():
        w = normal_bf16(g, (n, k), 0.02)
        b = normal_bf16(g, (n,), 0.01)
        q = oq.quantize(w, mode, 32 if mode == "mxfp8" else 64, bits)
        quant[name] = (q, b)
        p_oracle[f"{name}.weight"] = oq.dequantize(q, k)
        p_oracle[f"{name}.bias"] = b
    tables = {}
    for name, shape in table_specs(video, audio).items():
        t = normal_f32(g, shape, 0.1)
        if name.endswith("norm.weight"):
            t = (1.0 + t).astype(np.float32)
        tables[name] = t
        p_oracle[name] = t
    return p_oracle, quant, tables


def gpu_block(quant: dict, tables: dict, video, audio, mode: str):
    """``BasicAVTransformerBlock`` on cuda:0 over the arrays of ``block_params``."""
    import torch

    import ltxq
    from ltxq.block import BasicAVTransformerBlock

    lin = {}
    for name, (q, b) in quant.items():
        s = to_dev(q["scales"]) if mode == "affine" else torch.from_numpy(q["scales"].copy()).cuda()
        lin[name] = ltxq.QuantizedLinear(to_dev(q["weight"]), s, to_dev(q["biases"]) if mode == "affine" else None,
                                         to_dev_bf16(b), group_size=q["group_size"], bits=q["bits"], mode=mode)
    return BasicAVTransformerBlock(lin, {k: torch.from_numpy(v).cuda() for k, v in tables.items()}, video, audio)


def rope_np(g: np.random.Generator, heads: int, t: int, d: int):
    """Random RoPE (cos, sin) tables (heads, t, d / 2) fp32."""
    ang = g.uniform(0, 6.28, (heads, t, d // 2)).astype(np.float32)
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
