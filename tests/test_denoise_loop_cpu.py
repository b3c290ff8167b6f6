"""CPU test of ``ltxq.denoise.denoise_av``'s host logic: batching the
positive and negative passes into one call and slicing the velocities
back, the STG pass and its cutoff, the gradient-estimation history, masked
(per-token) timesteps and the mask blend, against the oracle loop
(av_pipeline.py:625-756).

Test doubles stand in for the GPU pieces: the velocity model is a CPU
function of the latent, timesteps, context and perturbation flag made of
fp32 multiplies and adds only (so numpy reproduces it bit for bit), and
``denoise_update`` is served by the oracle step (the CUDA kernel is
bit-identical to it; the GPU tests check that)."""

import numpy as np
import pytest
import torch

import ltxq.denoise as D
from helpers import normal_bf16, rng
from oracle import denoise as od
from oracle.bf16 import rbf16

C = 16  # latent channels of the test double


def _velocity_np(lat, ts, ctx, w, perturbed):
    t = ts[:, None, None] if ts.ndim == 1 else ts[:, :, None]
    v = ((lat * np.float32(w)).astype(np.float32) + ctx[:, :1, :C]).astype(np.float32)
    v = (v + t).astype(np.float32)
    return rbf16((v * np.float32(0.5)).astype(np.float32) if perturbed else v)


class FakeModel:
    """velocity = bf16((latent * w + context[:, 0, :C] + timesteps) [* 0.5 when perturbed])."""

    def __init__(self):
        self.calls = []

    def __call__(self, video, audio, shard=None, perturbations=None):
        self.calls.append((video.latent.shape[0], perturbations is not None))

        def vel(m, w):
            t = m.timesteps.float()
            t = t[:, None, None] if t.dim() == 1 else t[:, :, None]
            v = m.latent.float() * w + m.context.float()[:, :1, :C]
            v = v + t
            if perturbations is not None:
                v = v * 0.5
            return v.to(torch.bfloat16)

        return vel(video, 0.7), vel(audio, 1.3)


def _oracle_update_double(latent, v_cond, sigma, sigma_next, v_uncond=None, cfg_scale=1.0, v_perturbed=None,
                          stg_scale=0.0, denoise_mask=None, clean_latent=None, prev_velocity=None, ge_gamma=0.0,
                          have_prev=False, out=None):
    f = lambda t: None if t is None else t.float().numpy()  # noqa: E731
    new, cur = od.denoise_update(f(latent), f(v_cond), sigma, sigma_next, v_uncond=f(v_uncond), cfg_scale=cfg_scale,
                                 v_perturbed=f(v_perturbed), stg_scale=stg_scale, denoise_mask=f(denoise_mask),
                                 clean_latent=f(clean_latent),
                                 prev_velocity=f(prev_velocity) if have_prev else None, ge_gamma=ge_gamma)
    if ge_gamma > 0:
        prev_velocity.copy_(torch.from_numpy(cur))
    return torch.from_numpy(new).to(torch.bfloat16)


@pytest.mark.parametrize("cfg,stg,ge,masked", [(1.0, 0.0, 0.0, False), (3.0, 0.0, 0.0, False),
                                               (2.5, 1.0, 0.0, False), (3.0, 0.0, 1.5, False),
                                               (2.0, 0.5, 2.0, True), (1.0, 0.0, 0.0, True)])
def test_denoise_av_host_logic_matches_the_oracle_loop(monkeypatch, cfg, stg, ge, masked):
    from ltxq.perturbations import create_batched_stg_config

    monkeypatch.setattr(D, "denoise_update", _oracle_update_double)
    g = rng(int(cfg * 10 + stg * 7 + ge * 3) + masked)
    B, T, A, L = 2, 12, 5, 3
    vl, al = normal_bf16(g, (B, T, C)), normal_bf16(g, (B, A, C))
    vctx, actx, nvctx, nactx = (normal_bf16(g, (B, L, 24)) for _ in range(4))
    vmask = amask = vclean = aclean = None
    if masked:
        vmask = np.ones((B, T), np.float32)
        vmask[:, :3] = 0.0
        vmask[:, 3:5] = 0.5
        amask = np.ones((B, A), np.float32)
        amask[0, 0] = 0.0
        vclean, aclean = normal_bf16(g, (B, T, C)), normal_bf16(g, (B, A, C))
    sigmas = np.asarray(od.DISTILLED_SIGMA_VALUES[:5] + [0.0], np.float32)
    cutoff = 0.6

    def model_np(vlat, alat, vt, at, pass_):
        neg = pass_ == "negative"
        ptb = pass_ == "perturbed"
        return (_velocity_np(vlat, vt, nvctx if neg else vctx, 0.7, ptb),
                _velocity_np(alat, at, nactx if neg else actx, 1.3, ptb))

    ref_v, ref_a = od.denoise_loop_av_general(model_np, vl, al, sigmas, cfg, cfg if cfg == 1.0 else 1.5, stg, cutoff,
                                              ge, vmask, vclean, amask, aclean)
    t = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a))  # noqa: E731
    b16 = lambda a: None if a is None else t(a).to(torch.bfloat16)  # noqa: E731
    model = FakeModel()
    pe = (torch.zeros(1), torch.zeros(1))  # the double ignores RoPE
    fv, fa = D.denoise_av(model, D.LatentState(b16(vl), t(vmask), b16(vclean)),
                          D.LatentState(b16(al), t(amask), b16(aclean)), sigmas, b16(vctx), b16(actx), pe, pe, pe, pe,
                          negative_video_context=b16(nvctx), negative_audio_context=b16(nactx),
                          video_guider=D.CFGGuider(cfg), audio_guider=D.CFGGuider(cfg if cfg == 1.0 else 1.5),
                          ge_gamma=ge, stg_guider=D.STGGuider(stg) if stg else None,
                          stg_perturbations=create_batched_stg_config(B) if stg else None, stg_cutoff=cutoff)
    assert np.array_equal(fv.latent.float().numpy(), ref_v)
    assert np.array_equal(fa.latent.float().numpy(), ref_a)
    # per step: one pass (2B rows with CFG), then the batch-B perturbed pass while STG is on
    steps = len(sigmas) - 1
    expect = []
    for i in range(steps):
        expect.append((2 * B if cfg != 1.0 else B, False))
        if stg and (i + 1) / steps <= cutoff:
            expect.append((B, True))
    assert model.calls == expect


@pytest.mark.parametrize("cfg,stg,ge,masked", [(1.0, 0.0, 0.0, False), (3.0, 0.0, 0.0, False),
                                               (2.5, 1.0, 1.5, False), (2.0, 0.5, 2.0, True)])
def test_denoise_heun_av_matches_the_oracle_loop(cfg, stg, ge, masked):
    """The Heun loop (av_pipeline.py:758-897) with the same test double:
    predictor and corrector passes, guidance, gradient estimation, masks,
    and the last step leaving the fp32 X0 -- bit for bit against the oracle
    loop (all of its step arithmetic is torch fp32)."""
    from ltxq.perturbations import create_batched_stg_config

    g = rng(int(cfg * 10 + stg * 7 + ge * 3) + masked + 100)
    B, T, A, L = 2, 12, 5, 3
    vl, al = normal_bf16(g, (B, T, C)), normal_bf16(g, (B, A, C))
    vctx, actx, nvctx, nactx = (normal_bf16(g, (B, L, 24)) for _ in range(4))
    vmask = amask = vclean = aclean = None
    if masked:
        vmask = np.ones((B, T), np.float32)
        vmask[:, :4] = 0.0
        amask = np.ones((B, A), np.float32)
        amask[1, :2] = 0.25
        vclean, aclean = normal_bf16(g, (B, T, C)), normal_bf16(g, (B, A, C))
    sigmas = np.asarray([1.0, 0.909375, 0.725, 0.421875, 0.0], np.float32)
    cutoff = 0.5

    def model_np(vlat, alat, vt, at, pass_):
        neg = pass_ == "negative"
        ptb = pass_ == "perturbed"
        return (_velocity_np(vlat, vt, nvctx if neg else vctx, 0.7, ptb),
                _velocity_np(alat, at, nactx if neg else actx, 1.3, ptb))

    a_cfg = cfg if cfg == 1.0 else 1.5
    ref_v, ref_a = od.denoise_loop_heun_av(model_np, vl, al, sigmas, cfg, a_cfg, stg, cutoff, ge, vmask, vclean,
                                           amask, aclean)
    t = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a))  # noqa: E731
    b16 = lambda a: None if a is None else t(a).to(torch.bfloat16)  # noqa: E731
    model = FakeModel()
    pe = (torch.zeros(1), torch.zeros(1))
    fv, fa = D.denoise_heun_av(model, D.LatentState(b16(vl), t(vmask), b16(vclean)),
                               D.LatentState(b16(al), t(amask), b16(aclean)), sigmas, b16(vctx), b16(actx), pe, pe,
                               pe, pe, negative_video_context=b16(nvctx), negative_audio_context=b16(nactx),
                               video_guider=D.CFGGuider(cfg), audio_guider=D.CFGGuider(a_cfg), ge_gamma=ge,
                               stg_guider=D.STGGuider(stg) if stg else None,
                               stg_perturbations=create_batched_stg_config(B) if stg else None, stg_cutoff=cutoff)
    assert fv.latent.dtype == torch.float32  # the last step leaves the X0
    assert np.array_equal(fv.latent.numpy(), ref_v) and np.array_equal(fa.latent.numpy(), ref_a)
    # two transformer points per step but the last (predictor only), + the STG passes
    steps = len(sigmas) - 1
    n_main = 2 * steps - 1
    n_stg = sum(1 for i in range(steps) if stg and (i + 1) / steps <= cutoff)
    assert len(model.calls) == n_main + n_stg
