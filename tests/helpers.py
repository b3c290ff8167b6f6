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
