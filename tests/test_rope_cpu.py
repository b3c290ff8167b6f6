"""CPU tests of the RoPE tables and latent positions (``ltxq.rope``) against
the oracle restatement of LTX_2_MLX/model/transformer/rope.py and
components/patchifiers.py: positions bit for bit, the float64 frequency
grid bit for bit, the tables within fp32 cos / sin accuracy."""

import numpy as np
import pytest
import torch

from oracle import rope as orope


@pytest.mark.parametrize("frames,height,width,fps", [(3, 4, 5, 24.0), (2, 2, 3, 25.0), (5, 1, 2, 23.976)])
@pytest.mark.parametrize("causal", [True, False])
def test_video_positions(frames, height, width, fps, causal):
    from ltxq.rope import video_positions

    got = video_positions(2, frames, height, width, fps, causal_fix=causal)
    ref = orope.video_positions(2, frames, height, width, fps, causal_fix=causal)
    assert got.shape == (2, 3, frames * height * width, 2) and got.dtype == torch.float32
    assert np.array_equal(got.numpy().view(np.uint32), ref.view(np.uint32))
    # patch bounds: pixels for height / width, the causal first frame covers one video frame
    assert got[0, 1, 0].tolist() == [0.0, 32.0] and got[0, 2, 1].tolist() == [32.0, 64.0]
    if causal:
        assert got[0, 0, 0].tolist() == [0.0, np.float32(1.0) / np.float32(fps)]


@pytest.mark.parametrize("frames,shift", [(201, 0), (17, 3)])
def test_audio_positions(frames, shift):
    from ltxq.rope import audio_positions

    got = audio_positions(2, frames, shift=shift)
    ref = orope.audio_positions(2, frames, shift=shift)
    assert got.shape == (2, 1, frames, 2)
    assert np.array_equal(got.numpy().view(np.uint32), ref.view(np.uint32))
    assert got[0, 0, -1, 1] > got[0, 0, -1, 0]


@pytest.mark.parametrize("n_dims,dim", [(3, 4096), (1, 2048), (3, 1024)])
def test_double_frequency_grid(n_dims, dim):
    from ltxq.rope import freq_grid

    got = freq_grid(10000.0, n_dims, dim, double=True).numpy()
    ref = orope.freq_grid(10000.0, n_dims, dim, double=True)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    assert got[0] == np.float32(np.pi / 2) and abs(got[-1] / (10000.0 * np.pi / 2) - 1) < 1e-6


@pytest.mark.parametrize("double", [True, False])
def test_video_and_cross_tables(double):
    from ltxq.rope import AUDIO_MAX_POS, VIDEO_MAX_POS, precompute_freqs_cis, video_positions

    pos = video_positions(1, 3, 4, 5, 24.0)
    cos, sin = precompute_freqs_cis(pos, 4096, 10000.0, VIDEO_MAX_POS, True, 32, double)
    rc, rs = orope.precompute_freqs_cis(pos.numpy(), 4096, 10000.0, list(VIDEO_MAX_POS), True, 32, double)
    assert cos.shape == (1, 32, 60, 64) and cos.is_contiguous()
    # the double grid is exact (cos / sin within an fp32 ulp); the fp32 grid
    # may differ by an ulp of powf (4 of 682 values here), ~2.4e-4 at 15708 rad
    tol = 1e-6 if double else 1e-3
    assert np.max(np.abs(cos.numpy() - rc)) <= tol and np.max(np.abs(sin.numpy() - rs)) <= tol
    # 2046 frequencies fill 2048 slots: the first two (head 0's first two) are the identity
    assert torch.all(cos[:, 0, :, :2] == 1) and torch.all(sin[:, 0, :, :2] == 0)
    ccos, csin = precompute_freqs_cis(pos[:, 0:1], 2048, 10000.0, AUDIO_MAX_POS, True, 32, double)
    rcc, rcs = orope.precompute_freqs_cis(pos[:, 0:1].numpy(), 2048, 10000.0, list(AUDIO_MAX_POS), True, 32, double)
    assert ccos.shape == (1, 32, 60, 32)
    assert np.max(np.abs(ccos.numpy() - rcc)) <= tol and np.max(np.abs(csin.numpy() - rcs)) <= tol
    assert np.allclose(cos.numpy() ** 2 + sin.numpy() ** 2, 1.0, atol=1e-6)


def test_tables_rotate_like_the_reference_split_rope():
    """Driven through the split rotation (x1 cos - x2 sin, x1 sin + x2 cos
    per head, rope.py:38-90), the tables depend only on position: tokens at
    equal positions get equal tables, and the score of a query and a key at
    the same position does not depend on that position."""
    from ltxq.rope import AUDIO_MAX_POS, precompute_freqs_cis

    def rotate(x, cos, sin):
        x1, x2 = x.chunk(2, dim=-1)
        return torch.cat([x1 * cos - x2 * sin, x1 * sin + x2 * cos], dim=-1)

    grid = torch.tensor([[[[3.0, 3.0], [3.0, 3.0], [7.5, 7.5], [-2.0, -2.0]]]])  # (B=1, 1 dim, T=4, bounds)
    cos, sin = precompute_freqs_cis(grid, 64, 10000.0, AUDIO_MAX_POS, True, 2, True)
    assert torch.equal(cos[:, :, 0], cos[:, :, 1]) and torch.equal(sin[:, :, 0], sin[:, :, 1])
    g = torch.Generator().manual_seed(0)
    q = torch.randn(1, 2, 1, 32, generator=g, dtype=torch.float64).expand(1, 2, 4, 32)
    k = torch.randn(1, 2, 1, 32, generator=g, dtype=torch.float64).expand(1, 2, 4, 32)
    c, s_ = cos.double(), sin.double()
    scores = (rotate(q, c, s_) * rotate(k, c, s_)).sum(-1)
    assert torch.allclose(scores, scores[..., :1].expand_as(scores), atol=1e-9)


def test_positions_and_max_pos_must_agree():
    from ltxq.rope import precompute_freqs_cis

    with pytest.raises(ValueError):
        precompute_freqs_cis(torch.zeros(1, 3, 4, 2), 4096, max_pos=(20,), use_middle_indices_grid=True)
    with pytest.raises(ValueError):
        precompute_freqs_cis(torch.zeros(1, 1, 4), 64, max_pos=(20,), use_middle_indices_grid=True)
