"""Latent layouts and the Gaussian noiser's blend, restated in numpy (TEST
INFRASTRUCTURE ONLY; see the package docstring).

Follows LTX_2_MLX/components/patchifiers.py:52-122 (video, patch (1, p, p)),
:327-375 (audio) and components/noisers.py:57-75 (the fp32 two-step blend).
"""

from __future__ import annotations

import numpy as np

from .bf16 import rbf16

F32 = np.float32


def patchify_video(x, p: int = 1):
    b, c, f, h, w = x.shape
    x = x.reshape(b, c, f, 1, h // p, p, w // p, p).transpose(0, 2, 4, 6, 1, 3, 5, 7)
    return x.reshape(b, f * (h // p) * (w // p), c * p * p)


def unpatchify_video(t, c: int, f: int, h: int, w: int, p: int = 1):
    b = t.shape[0]
    x = t.reshape(b, f, h // p, w // p, c, 1, p, p).transpose(0, 4, 1, 5, 2, 6, 3, 7)
    return x.reshape(b, c, f, h, w)


def patchify_audio(x):
    b, c, t, f = x.shape
    return x.transpose(0, 2, 1, 3).reshape(b, t, c * f)


def noise_blend(latent, clean, mask, noise, scale: float):
    """clean + mask ((latent + s (noise - latent)) - clean) in fp32, then
    bf16 (the latent's dtype)."""
    base, cl, n = (np.asarray(a, F32) for a in (latent, clean, noise))
    m = np.asarray(mask, F32)[..., None]
    noised = (base + (F32(scale) * (n - base).astype(F32)).astype(F32)).astype(F32)
    return rbf16((cl + (m * (noised - cl).astype(F32)).astype(F32)).astype(F32))
