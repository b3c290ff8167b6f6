"""Denoise loop of the audio-video pipeline around ``LTXAVModel``.

Mirrors the reference's sampling components:

* sigma schedules: ``DISTILLED_SIGMA_VALUES`` / ``STAGE_2_DISTILLED_SIGMA_VALUES``
  and ``LTX2Scheduler`` (LTX_2_MLX/components/schedulers.py:13-140);
* ``CFGGuider`` / ``STGGuider`` (components/guiders.py:10-87), as scale
  holders with the reference's ``enabled()`` rules;
* ``denoise_update``: everything a step does after its transformer passes
  (velocity -> denoised, CFG, STG, gradient estimation, the denoise-mask
  blend, the Euler step; pipelines/av_pipeline.py:700-742) as ONE CUDA
  kernel launch per stream (``ltxq_denoise_update``), bit-identical to the
  reference's fp32 op sequence;
* ``denoise_av``: ``_denoise_loop_cfg_av`` (av_pipeline.py:625-756).  The
  positive and negative (CFG) passes run as one transformer pass over a
  batch of 2B: the weights stream from HBM once per step instead of twice.
  With ``graph=True`` the model call is captured once as a CUDA graph and
  replayed every step.

With an ``STGGuider`` and a ``BatchedPerturbationConfig``
(``ltxq.perturbations``), each step also runs the perturbed pass (the
positive inputs through blocks that skip the perturbed attention
sub-layers) until ``stg_cutoff`` of the steps, and the video update adds
the STG term after CFG, as av_pipeline.py:706-717 does.

``denoise_heun_av`` is ``_denoise_loop_heun_av`` (av_pipeline.py:758-897):
Euler predictor and Heun corrector in fp32 torch (``HeunDiffusionStep``).

Not built: the non-AV / two-stage pipelines.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass, replace

import numpy as np
import torch

from . import _lib
from .kernels import _require_cuda, _stream

DISTILLED_SIGMA_VALUES = (1.0, 0.99375, 0.9875, 0.98125, 0.975, 0.909375, 0.725, 0.421875, 0.0)
STAGE_2_DISTILLED_SIGMA_VALUES = (0.909375, 0.725, 0.421875, 0.0)
BASE_SHIFT_ANCHOR = 1024
MAX_SHIFT_ANCHOR = 4096


def ltx2_scheduler(steps: int, tokens: int | None = None, max_shift: float = 2.05, base_shift: float = 0.95,
                   stretch: bool = True, terminal: float = 0.1) -> np.ndarray:
    """LTX2Scheduler.execute (schedulers.py:20-95): fp32 sigmas (steps + 1,)
    shifted by the token count (``prod(latent.shape[2:])``, 4096 when not
    given) and stretched so that the last non-zero sigma is ``terminal``.
    Host arithmetic in fp32 with the reference's operation order."""
    f = np.float32
    tokens = MAX_SHIFT_ANCHOR if tokens is None else tokens
    n = steps + 1
    t = np.arange(n, dtype=f) / f(max(steps, 1))  # linspace(1, 0, n) = 1 * (1 - t) + 0 * t
    sig = (f(1.0) - t).astype(f)
    slope = (max_shift - base_shift) / (MAX_SHIFT_ANCHOR - BASE_SHIFT_ANCHOR)
    shift = math.exp(tokens * slope + (base_shift - slope * BASE_SHIFT_ANCHOR))
    nz = sig != 0
    out = np.zeros(n, dtype=f)
    out[nz] = f(shift) / (f(shift) + (f(1.0) / sig[nz] - f(1.0)))
    if stretch and steps > 0:
        # steps == 1 stretches by 0 (NaN first sigma), as the reference does
        one_minus = (f(1.0) - out).astype(f)
        scale = f(float(one_minus[steps - 1]) / (1.0 - terminal))
        keep = out != 0
        with np.errstate(divide="ignore", invalid="ignore"):
            out[keep] = f(1.0) - one_minus[keep] / scale
    return out.astype(f)


def sigma_schedule(num_steps: int, distilled: bool = False, tokens: int | None = None) -> np.ndarray:
    """get_sigma_schedule (schedulers.py:121-140)."""
    if distilled:
        return np.asarray(DISTILLED_SIGMA_VALUES, dtype=np.float32)
    return ltx2_scheduler(num_steps, tokens)


def to_velocity(sample: torch.Tensor, sigma, denoised: torch.Tensor) -> torch.Tensor:
    """(sample - denoised) / sigma in fp32 (core_utils.py:25-52)."""
    if not isinstance(sigma, torch.Tensor) and sigma == 0:
        raise ValueError("Sigma can't be 0.0")
    s = sigma.float() if isinstance(sigma, torch.Tensor) else sigma
    return (sample.float() - denoised.float()) / s


class EulerDiffusionStep:
    """EulerDiffusionStep.step (diffusion_steps.py:8-70): denoised + (sigma_next
    / sigma) (sample - denoised) in fp32, cast to the sample's dtype.  The
    denoise loop applies it inside ``ltxq_denoise_update``; this class serves
    callers holding denoised predictions."""

    def step(self, sample: torch.Tensor, denoised_sample: torch.Tensor, sigmas, step_index: int, *,
             sigma: float | None = None, sigma_next: float | None = None) -> torch.Tensor:
        sigma = float(sigmas[step_index]) if sigma is None else sigma
        sigma_next = float(sigmas[step_index + 1]) if sigma_next is None else sigma_next
        d = denoised_sample.float()
        out = d + (sigma_next / sigma) * (sample.float() - d)
        return out if sample.dtype == torch.float32 else out.to(sample.dtype)


class HeunDiffusionStep:
    """HeunDiffusionStep.step (diffusion_steps.py:72-130): the Euler
    predictor, and with the denoised prediction at the predicted point the
    average of the two velocities."""

    def step(self, sample: torch.Tensor, denoised_sample: torch.Tensor, sigmas, step_index: int,
             denoised_at_predicted: torch.Tensor | None = None) -> torch.Tensor:
        sig = torch.as_tensor(np.asarray(sigmas, dtype=np.float32))
        s, sn = sig[step_index], sig[step_index + 1]
        dt = float(sn - s)
        velocity = to_velocity(sample, s, denoised_sample)
        predicted = sample.float() + velocity * dt
        if denoised_at_predicted is None:
            return predicted.to(sample.dtype)
        v2 = to_velocity(predicted.to(sample.dtype), sn, denoised_at_predicted)
        avg = 0.5 * (velocity + v2.float())
        return (sample.float() + avg * dt).to(sample.dtype)


@dataclass(frozen=True)
class CFGGuider:
    """Classifier-free guidance: cond + (scale - 1) * (cond - uncond)
    (guiders.py:10-32).  ``guide`` works on denoised predictions (fp32 from
    ``X0Model``); ``denoise_av`` applies the same arithmetic inside
    ``ltxq_denoise_update``."""

    scale: float

    def delta(self, cond: torch.Tensor, uncond: torch.Tensor) -> torch.Tensor:
        return (self.scale - 1) * (cond - uncond)

    def guide(self, cond: torch.Tensor, uncond: torch.Tensor) -> torch.Tensor:
        return cond + self.delta(cond, uncond)

    def enabled(self) -> bool:
        return self.scale != 1.0


def projection_coef(to_project: torch.Tensor, project_onto: torch.Tensor) -> torch.Tensor:
    """Per-sample <a, b> / (|b|^2 + 1e-8), shape (B, 1) (guiders.py:174-192)."""
    b = to_project.shape[0]
    a, o = to_project.reshape(b, -1), project_onto.reshape(b, -1)
    return (a * o).sum(dim=1, keepdim=True) / ((o * o).sum(dim=1, keepdim=True) + 1e-8)


@dataclass(frozen=True)
class CFGStarRescalingGuider:
    """CFG with the unconditioned prediction rescaled onto the conditioned
    one (guiders.py:35-62): cond + (scale - 1) * (cond - coef * uncond).
    The per-sample coefficient is a reduction over the whole latent, so the
    fused update does not apply it; call ``guide`` on denoised predictions."""

    scale: float

    def delta(self, cond: torch.Tensor, uncond: torch.Tensor) -> torch.Tensor:
        coef = projection_coef(cond, uncond)
        coef = coef.view((coef.shape[0],) + (1,) * (uncond.dim() - 1))
        return (self.scale - 1) * (cond - coef * uncond)

    def guide(self, cond: torch.Tensor, uncond: torch.Tensor) -> torch.Tensor:
        return cond + self.delta(cond, uncond)

    def enabled(self) -> bool:
        return self.scale != 1.0


@dataclass(frozen=True)
class STGGuider:
    """Spatio-temporal guidance: pos + scale * (pos - perturbed)
    (guiders.py:64-87)."""

    scale: float

    def delta(self, pos_denoised: torch.Tensor, perturbed_denoised: torch.Tensor) -> torch.Tensor:
        return self.scale * (pos_denoised - perturbed_denoised)

    def guide(self, pos_denoised: torch.Tensor, perturbed_denoised: torch.Tensor) -> torch.Tensor:
        return pos_denoised + self.delta(pos_denoised, perturbed_denoised)

    def enabled(self) -> bool:
        return self.scale != 0.0


@dataclass
class LatentState:
    """One stream's latent (bf16 (B, T, 128)), its denoise mask (fp32
    (B, T), None = all tokens denoised) and the clean latent the mask blends
    back in (bf16, with a mask)."""

    latent: torch.Tensor
    denoise_mask: torch.Tensor | None = None
    clean_latent: torch.Tensor | None = None

    def timesteps(self, sigma: float) -> torch.Tensor:
        """``modality_from_state`` (pipelines/common.py:207-250): fp32 (B,)
        full of sigma for a uniform mask, else mask * sigma per token."""
        b = self.latent.shape[0]
        full = torch.full((b,), sigma, dtype=torch.float32, device=self.latent.device)
        if self.denoise_mask is None:
            return full
        return self.denoise_mask.float() * full[:, None]


def _bf16_3d(t: torch.Tensor, name: str) -> torch.Tensor:
    _require_cuda(t, name)
    if t.dtype != torch.bfloat16 or t.dim() != 3 or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous bf16 (B, T, C) tensor")
    return t


def denoise_update(latent: torch.Tensor, v_cond: torch.Tensor, sigma: float, sigma_next: float,
                   v_uncond: torch.Tensor | None = None, cfg_scale: float = 1.0,
                   v_perturbed: torch.Tensor | None = None, stg_scale: float = 0.0,
                   denoise_mask: torch.Tensor | None = None, clean_latent: torch.Tensor | None = None,
                   prev_velocity: torch.Tensor | None = None, ge_gamma: float = 0.0, have_prev: bool = False,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """The latent after one step, from the step's velocities (bf16 (B, T,
    C)); see ``ltxq_denoise_update``.  ``prev_velocity`` (fp32 (B, T, C)) is
    read when ``have_prev`` and overwritten with this step's velocity when
    ``ge_gamma > 0``.  ``out`` may be ``latent`` (in-place)."""
    latent = _bf16_3d(latent, "latent")
    shape = tuple(latent.shape)
    if v_cond is None:
        raise ValueError("v_cond is required")
    for t, name in ((v_cond, "v_cond"), (v_uncond, "v_uncond"), (v_perturbed, "v_perturbed"),
                    (clean_latent, "clean_latent"), (out, "out")):
        if t is not None and tuple(_bf16_3d(t, name).shape) != shape:
            raise ValueError(f"{name} shape {tuple(t.shape)} != latent shape {shape}")
    if denoise_mask is not None:
        _require_cuda(denoise_mask, "denoise_mask")
        if denoise_mask.dtype != torch.float32 or tuple(denoise_mask.shape) != shape[:2]:
            raise ValueError("denoise_mask must be fp32 (B, T)")
        denoise_mask = denoise_mask.contiguous()
    if prev_velocity is not None:
        _require_cuda(prev_velocity, "prev_velocity")
        if prev_velocity.dtype != torch.float32 or tuple(prev_velocity.shape) != shape or \
                not prev_velocity.is_contiguous():
            raise ValueError("prev_velocity must be a contiguous fp32 tensor of the latent's shape")
    if out is None:
        out = torch.empty_like(latent)
    p = _lib.DenoiseParams(float(sigma), float(sigma_next), float(cfg_scale), float(stg_scale), float(ge_gamma),
                           1 if have_prev else 0, 0)
    ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    _lib.check(_lib.load().ltxq_denoise_update(
        latent.data_ptr(), v_cond.data_ptr(), ptr(v_uncond), ptr(v_perturbed), ptr(denoise_mask), ptr(clean_latent),
        ptr(prev_velocity), shape[0], shape[1], shape[2], ctypes.byref(p), out.data_ptr(), _stream()),
        "denoise_update")
    return out


def _batch2(t):
    """[t; t] along the batch dimension (a tuple of tables element-wise)."""
    if isinstance(t, tuple):
        return tuple(_batch2(x) for x in t)
    return torch.cat([t, t], dim=0)


def denoise_av(model, video: LatentState, audio: LatentState, sigmas, video_context: torch.Tensor,
               audio_context: torch.Tensor, video_pe: tuple, audio_pe: tuple, video_cross_pe: tuple,
               audio_cross_pe: tuple, negative_video_context: torch.Tensor | None = None,
               negative_audio_context: torch.Tensor | None = None, video_guider: CFGGuider = CFGGuider(1.0),
               audio_guider: CFGGuider = CFGGuider(1.0), ge_gamma: float = 0.0, stg_guider: STGGuider | None = None,
               stg_perturbations=None, stg_cutoff: float = 1.0, shard=None, graph: bool = False,
               callback=None) -> tuple[LatentState, LatentState]:
    """``_denoise_loop_cfg_av`` (av_pipeline.py:625-756) over ``model`` (an
    ``LTXAVModel``): per step one transformer pass (2B rows when either
    guider is enabled: positive then negative contexts), then one
    ``denoise_update`` per stream.  Gradient estimation (``ge_gamma``)
    applies to the video stream, as in the reference.  The STG pass (when
    ``stg_guider`` is enabled and ``stg_perturbations`` given) is a separate
    batch-B pass: its blocks skip sub-layers for the whole batch.  With a row
    shard, ``video`` holds this rank's rows."""
    from .model import Modality

    for gd in (video_guider, audio_guider):
        if type(gd) is not CFGGuider:  # the fused update applies plain CFG only
            raise ValueError(f"denoise_av takes CFGGuider guiders, got {type(gd).__name__}")
    if stg_guider is not None and type(stg_guider) is not STGGuider:
        raise ValueError(f"denoise_av takes an STGGuider, got {type(stg_guider).__name__}")
    sig = np.asarray(sigmas, dtype=np.float32)
    steps = len(sig) - 1
    need_cfg = video_guider.enabled() or audio_guider.enabled()
    if need_cfg and (negative_video_context is None or negative_audio_context is None):
        raise ValueError("CFG needs the negative video and audio contexts")
    b = video.latent.shape[0]
    if need_cfg:
        vctx = torch.cat([video_context, negative_video_context])
        actx = torch.cat([audio_context, negative_audio_context])
        vpe, ape, vcpe, acpe = (_batch2(t) for t in (video_pe, audio_pe, video_cross_pe, audio_cross_pe))
    else:
        vctx, actx, vpe, ape, vcpe, acpe = video_context, audio_context, video_pe, audio_pe, video_cross_pe, \
            audio_cross_pe
    rep = 2 if need_cfg else 1
    dev = video.latent.device
    # the model's per-step inputs live in fixed buffers (what a captured graph reads)
    v_in = torch.empty((rep * b,) + tuple(video.latent.shape[1:]), dtype=torch.bfloat16, device=dev)
    a_in = torch.empty((rep * b,) + tuple(audio.latent.shape[1:]), dtype=torch.bfloat16, device=dev)
    vt_shape = (rep * b,) if video.denoise_mask is None else (rep * b, video.latent.shape[1])
    at_shape = (rep * b,) if audio.denoise_mask is None else (rep * b, audio.latent.shape[1])
    v_t = torch.empty(vt_shape, dtype=torch.float32, device=dev)
    a_t = torch.empty(at_shape, dtype=torch.float32, device=dev)
    v_s = torch.empty((rep * b,), dtype=torch.float32, device=dev)

    def run(v_in, a_in, v_t, a_t, v_s):
        return model(Modality(v_in, v_t, vctx, vpe, vcpe, sigma=v_s),
                     Modality(a_in, a_t, actx, ape, acpe, sigma=v_s), shard)

    def run_perturbed(v_in, a_in, v_t, a_t, v_s):
        return model(Modality(v_in, v_t, video_context, video_pe, video_cross_pe, sigma=v_s),
                     Modality(a_in, a_t, audio_context, audio_pe, audio_cross_pe, sigma=v_s), shard,
                     stg_perturbations)

    stg_on = stg_guider is not None and stg_guider.enabled() and stg_perturbations is not None
    prev = torch.empty(video.latent.shape, dtype=torch.float32, device=dev) if ge_gamma > 0 else None
    step_graph = stg_graph = None
    for i in range(steps):
        sigma, sigma_next = float(sig[i]), float(sig[i + 1])
        for dst, st in ((v_in, video), (a_in, audio)):
            for r in range(rep):
                dst[r * b:(r + 1) * b].copy_(st.latent)
        for dst, st in ((v_t, video), (a_t, audio)):
            ts = st.timesteps(sigma)
            for r in range(rep):
                dst[r * b:(r + 1) * b].copy_(ts)
        v_s.fill_(sigma)
        if graph:
            if step_graph is None:
                from .graph import StepGraph

                step_graph = StepGraph(run, v_in, a_in, v_t, a_t, v_s)
            vv, av = step_graph.replay()
        else:
            vv, av = run(v_in, a_in, v_t, a_t, v_s)
        vc, ac = vv[:b], av[:b]
        vu, au = (vv[b:], av[b:]) if need_cfg else (None, None)
        stg_active = stg_on and (i + 1) / steps <= stg_cutoff  # av_pipeline.py:706-711
        vp = None
        if stg_active:  # the positive rows of the input buffers, through the perturbed blocks
            pos = (v_in[:b], a_in[:b], v_t[:b], a_t[:b], v_s[:b])
            if graph:
                if stg_graph is None:
                    from .graph import StepGraph

                    stg_graph = StepGraph(run_perturbed, *pos)
                vp = stg_graph.replay()[0]
            else:
                vp = run_perturbed(*pos)[0]
        new_v = denoise_update(video.latent, vc, sigma, sigma_next, v_uncond=vu,
                               cfg_scale=video_guider.scale if need_cfg else 1.0, v_perturbed=vp,
                               stg_scale=stg_guider.scale if stg_active else 0.0,
                               denoise_mask=video.denoise_mask, clean_latent=video.clean_latent,
                               prev_velocity=prev, ge_gamma=ge_gamma, have_prev=i > 0)
        new_a = denoise_update(audio.latent, ac, sigma, sigma_next, v_uncond=au,
                               cfg_scale=audio_guider.scale if need_cfg else 1.0,
                               denoise_mask=audio.denoise_mask, clean_latent=audio.clean_latent)
        video, audio = replace(video, latent=new_v), replace(audio, latent=new_a)
        if callback is not None:
            callback(i + 1, steps)
    for gr in (step_graph, stg_graph):
        if gr is not None:
            gr.release()
    return video, audio


def post_process_latent(denoised: torch.Tensor, denoise_mask: torch.Tensor | None,
                        clean_latent: torch.Tensor | None) -> torch.Tensor:
    """denoised * mask + clean * (1 - mask) (pipelines/common.py:169-191);
    a None mask is the all-ones mask."""
    if denoise_mask is None:
        return denoised
    m = denoise_mask.to(denoised.dtype)
    m = m[..., None] if m.dim() == denoised.dim() - 1 else m
    return denoised * m + clean_latent * (1 - m)


def denoise_heun_av(model, video: LatentState, audio: LatentState, sigmas, video_context: torch.Tensor,
                    audio_context: torch.Tensor, video_pe: tuple, audio_pe: tuple, video_cross_pe: tuple,
                    audio_cross_pe: tuple, negative_video_context: torch.Tensor | None = None,
                    negative_audio_context: torch.Tensor | None = None, video_guider=CFGGuider(1.0),
                    audio_guider=CFGGuider(1.0), ge_gamma: float = 0.0, stg_guider: STGGuider | None = None,
                    stg_perturbations=None, stg_cutoff: float = 1.0, shard=None,
                    callback=None) -> tuple[LatentState, LatentState]:
    """``_denoise_loop_heun_av`` (av_pipeline.py:758-897): per step the
    guided X0 at the current point (CFG -- plain or ``CFGStarRescalingGuider``
    -- STG, gradient estimation, mask blend), the Euler predictor, the guided
    X0 at the predicted point (CFG, mask blend) and the Heun corrector
    (``HeunDiffusionStep``).  The positive and negative passes of each point
    run as one batch-2B transformer pass; the step arithmetic is fp32 torch
    (X0Model, guiders, steppers), as in the reference.  At sigma_next = 0 the
    latents become the fp32 X0, as the reference leaves them."""
    from .model import Modality, X0Model

    sig = np.asarray(sigmas, dtype=np.float32)
    steps = len(sig) - 1
    need_cfg = video_guider.enabled() or audio_guider.enabled()
    if need_cfg and (negative_video_context is None or negative_audio_context is None):
        raise ValueError("CFG needs the negative video and audio contexts")
    b = video.latent.shape[0]
    if need_cfg:
        vctx = torch.cat([video_context, negative_video_context])
        actx = torch.cat([audio_context, negative_audio_context])
        vpe, ape, vcpe, acpe = (_batch2(t) for t in (video_pe, audio_pe, video_cross_pe, audio_cross_pe))
    else:
        vctx, actx, vpe, ape, vcpe, acpe = video_context, audio_context, video_pe, audio_pe, video_cross_pe, \
            audio_cross_pe
    rep = 2 if need_cfg else 1
    stg_on = stg_guider is not None and stg_guider.enabled() and stg_perturbations is not None
    heun = HeunDiffusionStep()

    def guided(vlat, alat, sigma):
        """Guided X0 predictions of both streams at (vlat, alat, sigma), and
        the video timesteps of the point."""
        vt, at = video.timesteps(sigma), audio.timesteps(sigma)
        rv = lambda t: torch.cat([t] * rep) if rep > 1 else t  # noqa: E731
        vs = torch.full((rep * b,), sigma, dtype=torch.float32, device=vlat.device)
        vm = Modality(rv(vlat), rv(vt), vctx, vpe, vcpe, sigma=vs)
        am = Modality(rv(alat), rv(at), actx, ape, acpe, sigma=vs)
        dv, da = X0Model(model)(vm, am, shard)
        if need_cfg:
            dv = video_guider.guide(dv[:b], dv[b:])
            da = audio_guider.guide(da[:b], da[b:])
        return dv, da, vt, at

    prev = None
    for i in range(steps):
        sigma, sigma_next = float(sig[i]), float(sig[i + 1])
        x_v, x_a = video.latent, audio.latent
        dv, da, vt, at = guided(x_v, x_a, sigma)
        if stg_on and (i + 1) / steps <= stg_cutoff:
            vs = torch.full((b,), sigma, dtype=torch.float32, device=x_v.device)
            vm = Modality(x_v, vt, video_context, video_pe, video_cross_pe, sigma=vs)
            am = Modality(x_a, at, audio_context, audio_pe, audio_cross_pe, sigma=vs)
            dp, _ = X0Model(model)(vm, am, shard, stg_perturbations)
            dv = stg_guider.guide(dv, dp)
        if ge_gamma > 0 and sigma > 0:
            cur = (x_v.float() - dv) / sigma
            if prev is not None:
                total = ge_gamma * (cur - prev) + prev
                dv = x_v.float() - total * sigma
            prev = cur
        dv = post_process_latent(dv, video.denoise_mask, video.clean_latent)
        da = post_process_latent(da, audio.denoise_mask, audio.clean_latent)
        if sigma_next == 0:
            video, audio = replace(video, latent=dv), replace(audio, latent=da)
        else:
            s32 = torch.tensor(sig[i])
            dt = float(sig[i + 1] - sig[i])
            pred_v = (x_v.float() + to_velocity(x_v, s32, dv) * dt).to(x_v.dtype)
            pred_a = (x_a.float() + to_velocity(x_a, s32, da) * dt).to(x_a.dtype)
            dv2, da2, _, _ = guided(pred_v, pred_a, sigma_next)
            dv2 = post_process_latent(dv2, video.denoise_mask, video.clean_latent)
            da2 = post_process_latent(da2, audio.denoise_mask, audio.clean_latent)
            video = replace(video, latent=heun.step(x_v, dv, sig, i, denoised_at_predicted=dv2))
            audio = replace(audio, latent=heun.step(x_a, da, sig, i, denoised_at_predicted=da2))
        if callback is not None:
            callback(i + 1, steps)
    return video, audio
