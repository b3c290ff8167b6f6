"""RoPE tables and latent positions for the model's preprocess.

The reference's preprocessor builds the rotary tables from the tokens'
positions when the caller passes none (``_prepare_positional_embeddings``
model.py:256-283, ``_prepare_cross_positional_embeddings`` :392-417) with
``precompute_freqs_cis`` (model/transformer/rope.py:286-338, split type).
The positions come from the latent tools (components/patchifiers.py:125-225
and 265-310, conditioning/tools.py:60-76): [start, end) bounds of every
token, in pixels for height / width and in seconds for time.

Everything here is table arithmetic in torch (fp32, or a float64 frequency
grid), computed once per stage on the tensors' device; the per-step rotation
itself is ``ltxq_qk_norm_rope``.
"""

from __future__ import annotations

import math

import torch

VIDEO_MAX_POS = (20, 2048, 2048)  # LTXModel positional_embedding_max_pos default (model.py:615-616)
AUDIO_MAX_POS = (20,)             # AUDIO_CROSS_PE_MAX_POS (model.py:520), also the audio stream's max_pos
THETA = 10000.0


def freq_grid(theta: float, n_pos_dims: int, dim: int, double: bool, device=None) -> torch.Tensor:
    """theta ** linspace(0, 1, dim // (2 n_pos_dims)) * pi / 2 as fp32
    (rope.py:92-167); ``double`` evaluates it in float64 first, as the
    reference's ``use_double_precision`` path does."""
    n = dim // (2 * n_pos_dims)
    if n <= 0:
        return torch.zeros(0, dtype=torch.float32, device=device)
    if double:
        t = torch.arange(n, dtype=torch.float64, device=device) / max(n - 1, 1)
        return (torch.pow(torch.tensor(theta, dtype=torch.float64, device=device), t) * (math.pi / 2)).float()
    t = torch.arange(n, dtype=torch.float32, device=device) / max(n - 1, 1)
    return torch.pow(torch.tensor(theta, dtype=torch.float32, device=device), t) * (math.pi / 2)


def precompute_freqs_cis(indices_grid: torch.Tensor, dim: int, theta: float = THETA, max_pos=VIDEO_MAX_POS,
                         use_middle_indices_grid: bool = False, num_attention_heads: int = 32,
                         use_double_precision: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
    """(cos, sin), each fp32 (B, heads, T, dim / 2 / heads), contiguous:
    positions (B, n_dims, T) or bounds (B, n_dims, T, 2) scaled to [-1, 1]
    per dimension by ``max_pos``, times the frequency grid; the frequencies
    that do not fill ``dim / 2`` are padded at the front with the identity
    rotation (cos 1, sin 0)."""
    g = indices_grid.float()
    n_dims = g.shape[1]
    if len(max_pos) != n_dims:
        raise ValueError(f"{n_dims} position dimensions but max_pos has {len(max_pos)}")
    ind = freq_grid(theta, n_dims, dim, use_double_precision, g.device)
    if use_middle_indices_grid:
        if g.dim() != 4 or g.shape[-1] != 2:
            raise ValueError("use_middle_indices_grid needs (B, n_dims, T, 2) bounds")
        g = (g[..., 0] + g[..., 1]) / 2.0
    elif g.dim() == 4:
        g = g[..., 0]
    frac = torch.stack([g[:, i, :] / max_pos[i] for i in range(n_dims)], dim=-1)  # (B, T, n_dims)
    scaled = frac * 2 - 1
    freqs = ind[None, None, None, :] * scaled[..., None]  # (B, T, n_dims, n_freq)
    b, t = freqs.shape[:2]
    freqs = freqs.transpose(2, 3).reshape(b, t, -1)
    cos, sin = torch.cos(freqs), torch.sin(freqs)
    pad = dim // 2 - freqs.shape[-1]
    if pad < 0:
        raise ValueError(f"{freqs.shape[-1]} frequencies exceed dim / 2 = {dim // 2}")
    if pad:
        cos = torch.cat([torch.ones(b, t, pad, dtype=cos.dtype, device=cos.device), cos], dim=-1)
        sin = torch.cat([torch.zeros(b, t, pad, dtype=sin.dtype, device=sin.device), sin], dim=-1)
    cos = cos.reshape(b, t, num_attention_heads, -1).transpose(1, 2).contiguous()
    sin = sin.reshape(b, t, num_attention_heads, -1).transpose(1, 2).contiguous()
    return cos, sin


def video_positions(batch: int, frames: int, height: int, width: int, fps: float, scale=(8, 32, 32),
                    causal_fix: bool = True, device=None) -> torch.Tensor:
    """(B, 3, frames * height * width, 2) fp32 bounds of the latent tokens
    (patch size 1, frame-major order) in decoded-video units: pixels for
    height / width, seconds for time (the causal VAE's first latent frame
    covers one video frame)."""
    f, h, w = torch.meshgrid(torch.arange(frames, device=device), torch.arange(height, device=device),
                             torch.arange(width, device=device), indexing="ij")
    starts = torch.stack([f, h, w]).reshape(3, -1)
    coords = torch.stack([starts, starts + 1], dim=-1) * torch.tensor(scale, device=device).view(3, 1, 1)
    if causal_fix:
        coords[0] = torch.clamp(coords[0] + 1 - scale[0], min=0)
    pos = coords.float()
    pos[0] = pos[0] / fps
    return pos[None].expand(batch, -1, -1, -1).contiguous()


def audio_positions(batch: int, frames: int, sample_rate: int = 16000, hop_length: int = 160, downsample: int = 4,
                    is_causal: bool = True, shift: int = 0, device=None) -> torch.Tensor:
    """(B, 1, frames, 2) fp32 [start, end) times in seconds of the audio
    latent frames."""
    def times(a: int, b: int) -> torch.Tensor:
        mel = torch.arange(a, b, device=device).float() * downsample
        if is_causal:
            mel = torch.clamp(mel + 1 - downsample, min=0)
        return mel * hop_length / sample_rate

    pos = torch.stack([times(shift, frames + shift), times(shift + 1, frames + shift + 1)], dim=-1)
    return pos[None, None].expand(batch, 1, -1, -1).contiguous()
