"""CPU tests of the latent layouts and the Gaussian noiser (``ltxq.latents``)
against the oracle restatement of the reference's patchifiers and noiser."""

import numpy as np
import pytest
import torch

from helpers import normal_bf16, rng
from oracle import latents as ol


@pytest.mark.parametrize("shape,p", [((2, 128, 3, 4, 5), 1), ((1, 8, 2, 4, 6), 2)])
def test_video_patchify_round_trip(shape, p):
    from ltxq.latents import patchify_video, unpatchify_video

    x = torch.randn(*shape)
    tok = patchify_video(x, p)
    assert np.array_equal(tok.numpy(), ol.patchify_video(x.numpy(), p))
    b, c, f, h, w = shape
    assert tok.shape == (b, f * (h // p) * (w // p), c * p * p)
    assert torch.equal(unpatchify_video(tok, c, f, h, w, p), x)
    if p == 1:  # token order matches the positions' frame-major order
        assert torch.equal(tok[0, 1 * h * w + 2 * w + 3], x[0, :, 1, 2, 3])


def test_audio_patchify_round_trip():
    from ltxq.latents import patchify_audio, unpatchify_audio

    x = torch.randn(2, 8, 201, 16)
    tok = patchify_audio(x)
    assert tok.shape == (2, 201, 128) and np.array_equal(tok.numpy(), ol.patchify_audio(x.numpy()))
    assert torch.equal(unpatchify_audio(tok, 8, 16), x)


@pytest.mark.parametrize("scale", [1.0, 0.909375, 0.25])
def test_noiser_blend_matches_the_oracle(scale):
    from ltxq.denoise import LatentState
    from ltxq.latents import add_noise, initial_state

    g = rng(int(scale * 100))
    lat, clean, noise = (normal_bf16(g, (2, 10, 8)) for _ in range(3))
    mask = np.ones((2, 10), np.float32)
    mask[:, :3] = 0.0
    mask[1, 3:5] = 0.5
    b16 = lambda a: torch.from_numpy(a).to(torch.bfloat16)  # noqa: E731
    st = LatentState(b16(lat), torch.from_numpy(mask), b16(clean))
    got = add_noise(st, scale, noise=b16(noise))
    assert got.latent.dtype == torch.bfloat16
    assert np.array_equal(got.latent.float().numpy(), ol.noise_blend(lat, clean, mask, noise, scale))
    # conditioned tokens (mask 0) keep the clean latent
    assert torch.equal(got.latent[:, :3], b16(clean)[:, :3])
    # text-to-video start: zeros, full mask, scale 1 -> the noise itself
    init = initial_state(torch.zeros(1, 6, 8, dtype=torch.bfloat16))
    gen = torch.Generator().manual_seed(0)
    n = add_noise(init, 1.0, generator=gen)
    gen = torch.Generator().manual_seed(0)
    assert torch.equal(n.latent, torch.randn((1, 6, 8), generator=gen, dtype=torch.bfloat16))
