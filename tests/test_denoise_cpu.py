"""CPU tests of the denoise-loop host logic and its oracle: the sigma
schedules (the properties the reference's tests/test_scheduler.py checks,
and the ltxq host code against the oracle restatement bit for bit), and
identities of the oracle's fused step (components/diffusion_steps.py,
components/guiders.py, pipelines/common.py) that pin its op order."""

import numpy as np
import pytest

from helpers import normal_bf16, rng
from oracle import denoise as od
from oracle.bf16 import rbf16


@pytest.mark.parametrize("steps", [1, 2, 8, 10, 20, 25, 30, 40, 50])
@pytest.mark.parametrize("tokens", [None, 1024, 3456, 9216, 61152])
def test_ltx2_scheduler_matches_oracle(steps, tokens):
    from ltxq.denoise import ltx2_scheduler

    got = ltx2_scheduler(steps, tokens)
    ref = od.ltx2_sigmas(steps, 4096 if tokens is None else tokens)
    assert got.dtype == np.float32 and got.shape == (steps + 1,)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("steps", [10, 20, 30, 50])
def test_ltx2_scheduler_properties(steps):
    """tests/test_scheduler.py:20-105 of the reference: length, monotone,
    starts positive, ends at 0, within [0, 10]; and the stretch puts the last
    non-zero sigma at the terminal value."""
    from ltxq.denoise import ltx2_scheduler

    s = ltx2_scheduler(steps)
    assert len(s) == steps + 1
    assert np.all(s[:-1] >= s[1:])
    assert s[0] > 0 and s[-1] == 0.0
    assert np.all(s >= 0) and np.all(s <= 10)
    assert abs(float(s[-2]) - 0.1) < 1e-6
    assert np.array_equal(s, ltx2_scheduler(steps))


def test_distilled_schedules():
    """tests/test_scheduler.py:108-147: 9 and 4 values, decreasing, ending
    at exactly 0, stage 2 below stage 1."""
    from ltxq.denoise import DISTILLED_SIGMA_VALUES, STAGE_2_DISTILLED_SIGMA_VALUES, sigma_schedule

    assert list(DISTILLED_SIGMA_VALUES) == od.DISTILLED_SIGMA_VALUES
    assert list(STAGE_2_DISTILLED_SIGMA_VALUES) == od.STAGE_2_DISTILLED_SIGMA_VALUES
    for vals, n in ((DISTILLED_SIGMA_VALUES, 9), (STAGE_2_DISTILLED_SIGMA_VALUES, 4)):
        v = np.asarray(vals)
        assert len(v) == n and v[-1] == 0.0 and np.all(v[:-1] >= v[1:])
    assert max(STAGE_2_DISTILLED_SIGMA_VALUES[:-1]) < max(DISTILLED_SIGMA_VALUES[:-1])
    d = sigma_schedule(8, distilled=True)
    assert d.dtype == np.float32 and np.array_equal(d, np.asarray(DISTILLED_SIGMA_VALUES, np.float32))


def _inputs(shape, seed=0):
    g = rng(seed)
    return [normal_bf16(g, shape) for _ in range(4)]


def test_oracle_step_is_the_euler_lerp_of_the_x0():
    """No guidance: out = bf16(d + r (x - d)) with d = x - sigma v, the
    reference's X0Model then EulerDiffusionStep."""
    x, v, _, _ = _inputs((2, 40, 128))
    s, sn = 0.909375, 0.725
    got, cur = od.denoise_update(x, v, s, sn)
    d = (x - (np.float32(s) * v).astype(np.float32)).astype(np.float32)
    r = np.float32(sn / s)
    ref = rbf16((d + (r * (x - d).astype(np.float32)).astype(np.float32)).astype(np.float32))
    assert cur is None
    assert np.array_equal(got, ref)


def test_oracle_final_step_returns_the_x0():
    """sigma_next = 0 (the last step): the result is bf16 of the denoised
    sample (tests/test_scheduler.py:197-213 exercises this step)."""
    x, v, u, _ = _inputs((1, 64, 128), 1)
    got, _ = od.denoise_update(x, v, 0.421875, 0.0, v_uncond=u, cfg_scale=3.0)
    d = (x - (np.float32(0.421875) * v).astype(np.float32)).astype(np.float32)
    du = (x - (np.float32(0.421875) * u).astype(np.float32)).astype(np.float32)
    d = (d + (np.float32(2.0) * (d - du).astype(np.float32)).astype(np.float32)).astype(np.float32)
    assert np.array_equal(got, rbf16(d))
    assert np.all(np.isfinite(got))


def test_oracle_guidance_degenerate_cases():
    """CFG scale 1 and STG scale 0 are the unguided step; a full mask is the
    unmasked step; gradient estimation without history only records the
    velocity."""
    x, v, u, p = _inputs((2, 24, 64), 2)
    base, _ = od.denoise_update(x, v, 0.98125, 0.975)
    assert np.array_equal(od.denoise_update(x, v, 0.98125, 0.975, v_uncond=u, cfg_scale=1.0)[0], base)
    assert np.array_equal(od.denoise_update(x, v, 0.98125, 0.975, v_perturbed=p, stg_scale=0.0)[0], base)
    ones = np.ones((2, 24), np.float32)
    clean = normal_bf16(rng(3), (2, 24, 64))
    assert np.array_equal(od.denoise_update(x, v, 0.98125, 0.975, denoise_mask=ones, clean_latent=clean)[0], base)
    got, cur = od.denoise_update(x, v, 0.98125, 0.975, ge_gamma=2.0)
    assert np.array_equal(got, base)
    assert cur.shape == x.shape and cur.dtype == np.float32


def test_oracle_zero_mask_keeps_the_clean_latent_at_the_end():
    """mask 0 tokens take the clean latent as their denoised value; with
    sigma_next = 0 the result is the clean latent."""
    x, v, _, _ = _inputs((1, 32, 128), 4)
    clean = normal_bf16(rng(5), (1, 32, 128))
    mask = np.zeros((1, 32), np.float32)
    mask[:, 16:] = 1.0
    got, _ = od.denoise_update(x, v, 0.725, 0.0, denoise_mask=mask, clean_latent=clean)
    assert np.array_equal(got[:, :16], clean[:, :16])


def test_perturbation_config():
    """components/perturbations.py semantics: a block skips a sub-layer only
    when every sample is perturbed for it; blocks=None means every block."""
    from ltxq.perturbations import (BatchedPerturbationConfig, Perturbation, PerturbationConfig, PerturbationType,
                                    create_batched_stg_config)

    stg = create_batched_stg_config(2, blocks=[3, 5])
    assert stg.skipped(3) == frozenset({"skip_video_self_attn"}) and stg.skipped(4) == frozenset()
    every = create_batched_stg_config(1)
    assert all(every.skipped(i) == frozenset({"skip_video_self_attn"}) for i in range(48))
    mixed = BatchedPerturbationConfig([PerturbationConfig([Perturbation(PerturbationType.SKIP_V2A_CROSS_ATTN)]),
                                       PerturbationConfig.empty()])
    assert not mixed.all_in_batch(PerturbationType.SKIP_V2A_CROSS_ATTN, 0) and mixed.skipped(0) == frozenset()
    assert BatchedPerturbationConfig.empty(3).skipped(0) == frozenset()
    assert not create_batched_stg_config(1, skip_video_self_attn=False).skipped(0)


def test_guiders_match_the_oracle():
    """CFGGuider / STGGuider.guide on fp32 denoised predictions bit for bit
    (elementwise fp32), CFGStarRescalingGuider within the accumulation order
    of its per-sample reduction."""
    import torch

    from ltxq.denoise import CFGGuider, CFGStarRescalingGuider, STGGuider

    g = rng(11)
    c, u, p = (g.standard_normal((2, 40, 16)).astype(np.float32) for _ in range(3))
    tc, tu, tp = (torch.from_numpy(a) for a in (c, u, p))
    assert np.array_equal(CFGGuider(3.5).guide(tc, tu).numpy(), od.cfg_guide(c, u, 3.5))
    assert np.array_equal(STGGuider(1.25).guide(tc, tp).numpy(), od.stg_guide(c, p, 1.25))
    got = CFGStarRescalingGuider(4.0).guide(tc, tu).numpy()
    assert np.allclose(got, od.cfg_star_guide(c, u, 4.0), rtol=1e-5, atol=1e-5)
    assert CFGGuider(1.0).enabled() is False and STGGuider(0.0).enabled() is False
    assert np.array_equal(CFGGuider(1.0).guide(tc, tu).numpy(), c)  # scale 1: the conditioned prediction


def test_cfg_guide_is_the_fused_update_arithmetic():
    """The fused step's CFG (oracle denoise_update) equals CFGGuider.guide on
    the X0 predictions followed by the Euler step."""
    x, v, u, _ = _inputs((1, 20, 16), 12)
    s, sn = 0.975, 0.909375
    got, _ = od.denoise_update(x, v, s, sn, v_uncond=u, cfg_scale=2.5)
    d = od.cfg_guide(od._x0(x, np.float32(s), v), od._x0(x, np.float32(s), u), 2.5)
    r = np.float32(sn / s)
    ref = rbf16((d + (r * (x - d).astype(np.float32)).astype(np.float32)).astype(np.float32))
    assert np.array_equal(got, ref)


def test_denoise_av_rejects_guiders_the_fused_update_cannot_apply():
    from ltxq.denoise import CFGGuider, CFGStarRescalingGuider, LatentState, denoise_av

    with pytest.raises(ValueError):
        denoise_av(None, LatentState(None), LatentState(None), [1.0, 0.0], None, None, None, None, None, None,
                   video_guider=CFGStarRescalingGuider(3.0), audio_guider=CFGGuider(1.0))


def test_steppers_match_the_oracle():
    """EulerDiffusionStep / HeunDiffusionStep on a bf16 sample and fp32
    denoised predictions, bit for bit; the reference's stepper tests
    (shapes kept, finite values, sigma_next = 0 handled) hold."""
    import torch

    from ltxq.denoise import EulerDiffusionStep, HeunDiffusionStep, to_velocity

    g = rng(13)
    x = normal_bf16(g, (2, 33, 16))
    d, d2 = (g.standard_normal((2, 33, 16)).astype(np.float32) for _ in range(2))
    tx = torch.from_numpy(x).to(torch.bfloat16)
    td, td2 = torch.from_numpy(d), torch.from_numpy(d2)
    sig = np.asarray(od.DISTILLED_SIGMA_VALUES, np.float32)
    for i in (0, 5, 7):  # step 7 ends at sigma 0
        got = EulerDiffusionStep().step(tx, td, sig, i)
        assert got.dtype == torch.bfloat16 and got.shape == tx.shape
        assert np.array_equal(got.float().numpy(), od.euler_step(x, d, float(sig[i]), float(sig[i + 1])))
    for i in (0, 5):
        h1 = HeunDiffusionStep().step(tx, td, sig, i)
        assert np.array_equal(h1.float().numpy(), od.heun_step(x, d, sig[i], sig[i + 1]))
        h2 = HeunDiffusionStep().step(tx, td, sig, i, denoised_at_predicted=td2)
        assert np.array_equal(h2.float().numpy(), od.heun_step(x, d, sig[i], sig[i + 1], d2))
        assert torch.isfinite(h2.float()).all()
    with pytest.raises(ValueError):
        to_velocity(tx, 0.0, td)
