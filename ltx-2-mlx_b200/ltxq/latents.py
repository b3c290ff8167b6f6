"""Latent formats either side of the model: the VAE latents <-> token
sequences (the reference's patchifiers, LTX_2_MLX/components/
patchifiers.py:14-122 and 221-375), the initial latent state
(conditioning/tools.py:37-80, 179-214) and the Gaussian noiser
(components/noisers.py:8-75).

Layout only, plus the noiser's fp32 blend; torch on the tensors' device.
The noise itself comes from torch's generator, so a seed does not give the
reference's MLX noise.
"""

from __future__ import annotations

import torch

from .denoise import LatentState


def patchify_video(latents: torch.Tensor, patch: int = 1) -> torch.Tensor:
    """(B, C, F, H, W) -> (B, F * (H/p) * (W/p), C * p * p): tokens in
    frame-major order, the channels (and the p x p patch) of each token
    contiguous (patchifiers.py:52-80)."""
    b, c, f, h, w = latents.shape
    x = latents.reshape(b, c, f, 1, h // patch, patch, w // patch, patch)
    x = x.permute(0, 2, 4, 6, 1, 3, 5, 7)
    return x.reshape(b, f * (h // patch) * (w // patch), c * patch * patch)


def unpatchify_video(tokens: torch.Tensor, channels: int, frames: int, height: int, width: int,
                     patch: int = 1) -> torch.Tensor:
    """The inverse of ``patchify_video`` (patchifiers.py:82-122)."""
    b = tokens.shape[0]
    x = tokens.reshape(b, frames, height // patch, width // patch, channels, 1, patch, patch)
    x = x.permute(0, 4, 1, 5, 2, 6, 3, 7)
    return x.reshape(b, channels, frames, height, width)


def patchify_audio(latents: torch.Tensor) -> torch.Tensor:
    """(B, C, T, F) -> (B, T, C * F) (patchifiers.py:327-345)."""
    b, c, t, f = latents.shape
    return latents.permute(0, 2, 1, 3).reshape(b, t, c * f)


def unpatchify_audio(tokens: torch.Tensor, channels: int, mel_bins: int) -> torch.Tensor:
    """(B, T, C * F) -> (B, C, T, F) (patchifiers.py:347-375)."""
    b, t, _ = tokens.shape
    return tokens.reshape(b, t, channels, mel_bins).permute(0, 2, 1, 3)


def initial_state(tokens: torch.Tensor) -> LatentState:
    """``create_initial_state`` (tools.py:37-80, 179-214) for patchified
    tokens: the latent and the clean latent are the given tokens (zeros for
    text-to-video), the denoise mask all ones -- held as None, the uniform
    mask, which gives the same values (timesteps sigma * 1 = sigma, blend
    d * 1 + clean * 0 = d) on the loop's broadcast-timestep path, as the
    reference's ``uniform_mask`` shortcut does (pipelines/common.py:231-240)."""
    return LatentState(tokens, None, tokens)


def add_noise(state: LatentState, noise_scale: float = 1.0, noise: torch.Tensor | None = None,
              generator: torch.Generator | None = None) -> LatentState:
    """GaussianNoiser.__call__ (noisers.py:29-75), in fp32:
    noised = latent + s (noise - latent); latent' = clean + mask (noised -
    clean), cast to the latent's dtype.  ``noise`` (in the latent's dtype)
    defaults to a standard normal draw from ``generator``.  A missing mask
    is all ones, a missing clean latent is the latent."""
    lat = state.latent
    if noise is None:
        noise = torch.randn(lat.shape, generator=generator, dtype=lat.dtype, device=lat.device)
    base = lat.float()
    clean = state.clean_latent.float() if state.clean_latent is not None else base
    mask = state.denoise_mask
    if mask is None:
        mask = torch.ones(lat.shape[:2], dtype=torch.float32, device=lat.device)
    m = mask.float()
    m = m[..., None] if m.dim() == lat.dim() - 1 else m
    noised = base + noise_scale * (noise.float() - base)
    out = clean + m * (noised - clean)
    return LatentState(out.to(lat.dtype), state.denoise_mask, state.clean_latent)
