"""RoPE table precompute and latent positions, restated in numpy (TEST
INFRASTRUCTURE ONLY; see the package docstring).

Follows LTX_2_MLX/model/transformer/rope.py:92-338 (``generate_freq_grid``,
``generate_freq_grid_float64_cpu``, ``generate_freqs``, ``split_freqs_cis``,
``precompute_freqs_cis``), components/patchifiers.py:125-225 and 265-310
(video patch bounds, pixel coordinates with the causal fix, audio timings)
and conditioning/tools.py:60-76 (temporal positions in seconds).  fp32
array math is one IEEE rounding per op; ``linspace(0, 1, n)`` is i / (n - 1)
(MLX's lerp form with start 0 and stop 1).  cos / sin / pow are evaluated
in float64 and rounded once to float32 (the reference's fp32 ``mx.cos`` may
differ by an ulp: parity within tolerance).
"""

from __future__ import annotations

import math

import numpy as np

F32 = np.float32


def freq_grid(theta: float, n_pos_dims: int, dim: int, double: bool) -> np.ndarray:
    """generate_freq_grid / generate_freq_grid_float64_cpu (rope.py:92-167):
    theta ** linspace(0, 1, dim // (2 n_pos_dims)) * pi / 2, fp32."""
    n = dim // (2 * n_pos_dims)
    if n <= 0:
        return np.zeros(0, F32)
    if double:
        t = np.arange(n, dtype=np.float64) / np.float64(max(n - 1, 1))
        return (np.power(np.float64(theta), t) * np.float64(math.pi / 2)).astype(F32)
    t = (np.arange(n, dtype=F32) / F32(max(n - 1, 1))).astype(F32)
    ind = np.power(np.float64(F32(theta)), t.astype(np.float64)).astype(F32)
    return (ind * F32(math.pi / 2)).astype(F32)


def precompute_freqs_cis(grid, dim: int, theta: float = 10000.0, max_pos=None, use_middle: bool = False,
                         heads: int = 32, double: bool = False):
    """precompute_freqs_cis (rope.py:286-338), split type: (cos, sin), each
    fp32 (B, heads, T, dim / 2 / heads), identity-padded at the front."""
    max_pos = [20, 2048, 2048] if max_pos is None else max_pos
    g = np.asarray(grid, F32)
    n_dims = g.shape[1]
    ind = freq_grid(theta, n_dims, dim, double)
    if use_middle:
        g = ((g[..., 0] + g[..., 1]).astype(F32) / F32(2.0)).astype(F32)
    elif g.ndim == 4:
        g = g[..., 0]
    frac = np.stack([(g[:, i, :] / F32(max_pos[i])).astype(F32) for i in range(n_dims)], axis=-1)
    scaled = ((frac * F32(2)).astype(F32) - F32(1)).astype(F32)
    freqs = (ind[None, None, None, :] * scaled[..., None]).astype(F32)  # (B, T, n_dims, n_freq)
    b, t = freqs.shape[:2]
    freqs = freqs.transpose(0, 1, 3, 2).reshape(b, t, -1)
    cos = np.cos(freqs.astype(np.float64)).astype(F32)
    sin = np.sin(freqs.astype(np.float64)).astype(F32)
    pad = dim // 2 - freqs.shape[-1]
    if pad:
        cos = np.concatenate([np.ones((b, t, pad), F32), cos], axis=-1)
        sin = np.concatenate([np.zeros((b, t, pad), F32), sin], axis=-1)
    cos = cos.reshape(b, t, heads, -1).transpose(0, 2, 1, 3)
    sin = sin.reshape(b, t, heads, -1).transpose(0, 2, 1, 3)
    return np.ascontiguousarray(cos), np.ascontiguousarray(sin)


def video_positions(batch: int, frames: int, height: int, width: int, fps: float, scale=(8, 32, 32),
                    causal_fix: bool = True) -> np.ndarray:
    """(B, 3, frames * height * width, 2) fp32 [start, end) bounds of every
    latent token (patch size 1), in pixels (frames: seconds), token order
    frame-major (patchifiers.py:125-178, 180-225; tools.py:60-76)."""
    f, h, w = np.meshgrid(np.arange(frames), np.arange(height), np.arange(width), indexing="ij")
    starts = np.stack([f, h, w]).reshape(3, -1)
    coords = np.stack([starts, starts + 1], axis=-1) * np.asarray(scale).reshape(3, 1, 1)
    if causal_fix:
        coords[0] = np.maximum(coords[0] + 1 - scale[0], 0)
    pos = coords.astype(F32)
    pos[0] = (pos[0] / F32(fps)).astype(F32)
    return np.broadcast_to(pos[None], (batch,) + pos.shape).copy()


def audio_positions(batch: int, frames: int, sample_rate: int = 16000, hop_length: int = 160, downsample: int = 4,
                    is_causal: bool = True, shift: int = 0) -> np.ndarray:
    """(B, 1, frames, 2) fp32 [start, end) times in seconds of every audio
    latent frame (patchifiers.py:265-310)."""
    def times(a, b):
        mel = (np.arange(a, b).astype(F32) * F32(downsample)).astype(F32)
        if is_causal:
            mel = np.maximum(((mel + F32(1)).astype(F32) - F32(downsample)).astype(F32), F32(0))
        return ((mel * F32(hop_length)).astype(F32) / F32(sample_rate)).astype(F32)

    pos = np.stack([times(shift, frames + shift), times(shift + 1, frames + shift + 1)], axis=-1)
    return np.broadcast_to(pos[None, None], (batch, 1, frames, 2)).copy()
