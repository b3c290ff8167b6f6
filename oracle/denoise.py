"""CPU oracle for the callers around the block loop: the model's input and
output stages and one denoise step (TEST INFRASTRUCTURE ONLY; see the
package docstring).

Restates, in numpy fp32 with the reference's rounding points:

* the sigma schedules (LTX_2_MLX/components/schedulers.py:13-140);
* the sinusoidal timestep embedding and the AdaLN MLP
  (model/transformer/timestep_embedding.py:8-201).  Their inputs are fp32,
  so MLX promotes the bf16 weights and the MLP runs in fp32;
* the velocity -> denoised conversion (model/transformer/model.py:1489-1540,
  ``X0Model``), the CFG / STG guiders (components/guiders.py:10-87), the
  gradient-estimation velocity blend and the mask blend of the AV CFG loop
  (pipelines/av_pipeline.py:700-742, pipelines/common.py:169-204), and the
  Euler step (components/diffusion_steps.py:19-70);
* the video / audio output head (model/transformer/model.py:1312-1340).

Every fp32 operation below is one IEEE round-to-nearest operation, as in
MLX's elementwise kernels.  A Python float scalar meets an fp32 array as an
fp32 value (MLX's weak scalar promotion), so scalar factors are rounded to
fp32 once, after their double-precision arithmetic.
"""

from __future__ import annotations

import math

import numpy as np

from .bf16 import rbf16
from .ref_ops import adaln

F32 = np.float32

# components/schedulers.py:100-118
DISTILLED_SIGMA_VALUES = [1.0, 0.99375, 0.9875, 0.98125, 0.975, 0.909375, 0.725, 0.421875, 0.0]
STAGE_2_DISTILLED_SIGMA_VALUES = [0.909375, 0.725, 0.421875, 0.0]


def ltx2_sigmas(steps: int, tokens: int = 4096, max_shift: float = 2.05, base_shift: float = 0.95,
                stretch: bool = True, terminal: float = 0.1) -> np.ndarray:
    """LTX2Scheduler.execute (schedulers.py:20-95), fp32 array math: linspace
    in fp32, shift from a linear fit on the token count, sigmoid-like
    transform, stretch so that the last non-zero sigma equals ``terminal``."""
    # mx.linspace(1, 0, n) as MLX's lerp form start * (1 - t) + stop * t with
    # t = i / (n - 1) in fp32 (ends exactly at 1 and 0; the interior values'
    # last bit is not pinned by a reference test)
    t = (np.arange(steps + 1, dtype=F32) / F32(max(steps, 1))).astype(F32)
    sig = (F32(1.0) - t).astype(F32)
    mm = (max_shift - base_shift) / (4096 - 1024)
    b = base_shift - mm * 1024
    exp_shift = F32(math.exp(tokens * mm + b))
    with np.errstate(divide="ignore"):
        inv = np.where(sig != 0, F32(1.0) / sig, F32(0.0)).astype(F32) - F32(1.0)
    tr = np.where(sig != 0, exp_shift / (exp_shift + inv), F32(0.0)).astype(F32)
    if stretch and steps > 0:
        om = (F32(1.0) - tr).astype(F32)
        last = float(om[steps - 1])
        factor = F32(last / (1.0 - terminal))
        with np.errstate(divide="ignore", invalid="ignore"):
            st = (F32(1.0) - om / factor).astype(F32)
        tr = np.where(tr != 0, st, tr).astype(F32)
    return tr.astype(F32)


def timestep_embedding(t, dim: int = 256, max_period: int = 10000) -> np.ndarray:
    """get_timestep_embedding with flip_sin_to_cos=True, shift 0, scale 1
    (timestep_embedding.py:8-58, Timesteps :61-84): [cos | sin] of t * freq."""
    half = dim // 2
    expo = (F32(-math.log(max_period)) * np.arange(half, dtype=F32)).astype(F32) / F32(half)
    freq = np.exp(expo.astype(np.float64)).astype(F32)
    arg = (np.asarray(t, dtype=F32)[:, None] * freq[None, :]).astype(F32)
    s = np.sin(arg.astype(np.float64)).astype(F32)
    c = np.cos(arg.astype(np.float64)).astype(F32)
    return np.concatenate([c, s], axis=-1)


def _silu(x):
    x = x.astype(np.float64)
    return (x / (1.0 + np.exp(-x))).astype(F32)


def _linear_f32(x, w, b):
    return (x.astype(np.float64) @ np.asarray(w, np.float64).T + np.asarray(b, np.float64)).astype(F32)


def ada_single(p: dict, t) -> tuple[np.ndarray, np.ndarray]:
    """AdaLayerNormSingle (timestep_embedding.py:165-201) on fp32 timesteps:
    (emb [N, n*D], embedded_timestep [N, D]), both fp32.  ``p`` holds
    linear_1 / linear_2 / linear weights and biases (bf16 values)."""
    h = timestep_embedding(t)
    h = _linear_f32(h, p["linear_1.weight"], p["linear_1.bias"])
    h = _silu(h)
    emb_t = _linear_f32(h, p["linear_2.weight"], p["linear_2.bias"])
    out = _linear_f32(_silu(emb_t), p["linear.weight"], p["linear.bias"])
    return out, emb_t


def linear_bf16(x, w, b):
    """bf16 nn.Linear: fp32 accumulation, one rounding."""
    return rbf16(_linear_f32(x, w, b))


def output_head(x, table, embedded, w, b, eps: float = 1e-6):
    """_process_video_output / _process_audio_output (model.py:1312-1340):
    shift/scale = bf16(table + embedded_timestep); LayerNorm (no affine,
    bf16 out); x * (1 + scale) + shift in bf16 ops; proj_out.  ``x`` [B, T,
    D] bf16 values, ``embedded`` [B, 1, D] fp32."""
    ss = rbf16((np.asarray(table, F32)[None, None] + np.asarray(embedded, F32)[:, :, None, :]).astype(F32))
    y = adaln(x, ss[:, :, 1], ss[:, :, 0], eps, norm="layer", vec_bf16=True)
    return linear_bf16(y, w, b)


def _x0(x, ts, v):
    """X0Model.denoise (model.py:1519-1525): latent - timesteps * velocity."""
    return (x - (ts * v).astype(F32)).astype(F32)


def denoise_update(latent, v_cond, sigma: float, sigma_next: float, v_uncond=None, cfg_scale: float = 1.0,
                   v_perturbed=None, stg_scale: float = 0.0, denoise_mask=None, clean_latent=None,
                   prev_velocity=None, ge_gamma: float = 0.0):
    """One step of the AV CFG loop for one stream (av_pipeline.py:700-742):
    X0 of each pass, CFG, STG, gradient estimation, mask blend, Euler step.
    Arrays are [B, T, C] (bf16 values as fp32); ``denoise_mask`` [B, T] fp32.
    Returns (new latent as bf16 values, this step's velocity or None)."""
    x = np.asarray(latent, F32)
    sig = F32(sigma)
    ts = sig if denoise_mask is None else (np.asarray(denoise_mask, F32) * sig).astype(F32)[..., None]
    d = _x0(x, ts, np.asarray(v_cond, F32))
    if v_uncond is not None and cfg_scale != 1.0:  # CFGGuider.guide (guiders.py:24-28)
        u = _x0(x, ts, np.asarray(v_uncond, F32))
        d = (d + (F32(cfg_scale - 1.0) * (d - u).astype(F32)).astype(F32)).astype(F32)
    if v_perturbed is not None and stg_scale != 0.0:  # STGGuider.guide (guiders.py:79-83)
        pt = _x0(x, ts, np.asarray(v_perturbed, F32))
        d = (d + (F32(stg_scale) * (d - pt).astype(F32)).astype(F32)).astype(F32)
    cur = None
    if ge_gamma > 0 and sigma > 0:  # av_pipeline.py:719-725
        cur = ((x - d).astype(F32) / sig).astype(F32)
        if prev_velocity is not None:
            total = ((F32(ge_gamma) * (cur - prev_velocity).astype(F32)).astype(F32) + prev_velocity).astype(F32)
            d = (x - (total * sig).astype(F32)).astype(F32)
    if denoise_mask is not None:  # post_process_latent (common.py:169-191)
        m = np.asarray(denoise_mask, F32)[..., None]
        clean = np.asarray(clean_latent, F32)
        d = ((d * m).astype(F32) + (clean * (F32(1.0) - m).astype(F32)).astype(F32)).astype(F32)
    ratio = F32(float(sigma_next) / float(sigma))  # EulerDiffusionStep.step (diffusion_steps.py:62-68)
    out = (d + (ratio * (x - d).astype(F32)).astype(F32)).astype(F32)
    return rbf16(out), cur


# non-block module prefixes of the reference model (model/transformer/model.py:640-712)
MODEL_PREFIXES = {
    "video": dict(patchify="patchify_proj", adaln="adaln_single", prompt="prompt_adaln_single",
                  cross_ss="av_ca_video_scale_shift_adaln_single", cross_gate="av_ca_a2v_gate_adaln_single",
                  table="scale_shift_table", proj_out="proj_out"),
    "audio": dict(patchify="audio_patchify_proj", adaln="audio_adaln_single", prompt="audio_prompt_adaln_single",
                  cross_ss="av_ca_audio_scale_shift_adaln_single", cross_gate="av_ca_v2a_gate_adaln_single",
                  table="audio_scale_shift_table", proj_out="audio_proj_out"),
}


def _ada_params(mp: dict, prefix: str) -> dict:
    return {"linear_1.weight": mp[f"{prefix}.emb.timestep_embedder.linear_1.weight"],
            "linear_1.bias": mp[f"{prefix}.emb.timestep_embedder.linear_1.bias"],
            "linear_2.weight": mp[f"{prefix}.emb.timestep_embedder.linear_2.weight"],
            "linear_2.bias": mp[f"{prefix}.emb.timestep_embedder.linear_2.bias"],
            "linear.weight": mp[f"{prefix}.linear.weight"], "linear.bias": mp[f"{prefix}.linear.bias"]}


def _prepare(mp: dict, which: str, s: dict, cross_sigma: float, ts_mult: float, av_ca_mult: float):
    """MultiModalTransformerArgsPreprocessor.prepare (model.py:285-340,
    445-505) for one batch row: timesteps uniform (= sigma) or per token
    (``s["timesteps"]`` (T,) fp32, the denoise mask times sigma)."""
    p = MODEL_PREFIXES[which]
    d = np.asarray(mp[f"{p['patchify']}.weight"]).shape[0]
    sig = (np.array([s["sigma"]], F32) * F32(ts_mult)).astype(F32)
    per_token = s.get("timesteps") is not None
    scaled = (np.asarray(s["timesteps"], F32) * F32(ts_mult)).astype(F32) if per_token else sig
    emb, emb_t = ada_single(_ada_params(mp, p["adaln"]), scaled)
    prompt, _ = ada_single(_ada_params(mp, p["prompt"]), sig)
    css, _ = ada_single(_ada_params(mp, p["cross_ss"]), scaled)
    cg, _ = ada_single(_ada_params(mp, p["cross_gate"]),
                       (np.array([cross_sigma], F32) * F32(av_ca_mult)).astype(F32))
    x = linear_bf16(s["latent"], mp[f"{p['patchify']}.weight"], mp[f"{p['patchify']}.bias"])
    lead = (-1,) if per_token else ()
    args = {"x": x, "context": s["context"], "timesteps": emb.reshape(lead + (9, d)), "pe": s["pe"],
            "cross_pe": s["cross_pe"], "cross_ss": css.reshape(lead + (4, d)), "cross_gate": cg.reshape(1, d),
            "prompt": prompt.reshape(2, d)}
    return args, emb_t


def model_forward(blocks_p: list, mp: dict, video: dict, audio: dict, heads_v: int, heads_a: int,
                  ts_mult: float = 1000.0, av_ca_mult: float = 1000.0, eps: float = 1e-6, skips=None):
    """LTXModel.__call__ (model.py:1344-1487) for one batch row: preprocess
    both streams, the blocks (``oracle.block.block``), the output heads.
    ``video`` / ``audio``: latent (T, 128) bf16 values, sigma (float),
    optional per-token timesteps (T,), context, pe, cross_pe.  Returns the
    (video, audio) velocities.  ``skips``: block index -> the sub-layers a
    perturbed (STG) pass skips there."""
    from .block import block

    va, vt = _prepare(mp, "video", video, audio["sigma"], ts_mult, av_ca_mult)
    aa, at = _prepare(mp, "audio", audio, video["sigma"], ts_mult, av_ca_mult)
    for i, p in enumerate(blocks_p):
        skip = (skips or {}).get(i, frozenset())
        vx, ax = block(p, va, aa, heads_v=heads_v, heads_a=heads_a, eps=eps, skip=skip)
        va, aa = dict(va, x=vx), dict(aa, x=ax)
    outs = []
    for which, args, emb_t in (("video", va, vt), ("audio", aa, at)):
        p = MODEL_PREFIXES[which]
        outs.append(output_head(args["x"][None], mp[p["table"]], emb_t[None], mp[f"{p['proj_out']}.weight"],
                                mp[f"{p['proj_out']}.bias"], eps)[0])
    return outs[0], outs[1]


def denoise_loop_av(model_fn, video_latent, audio_latent, sigmas, cfg_video: float = 1.0, cfg_audio: float = 1.0,
                    stg_scale: float = 0.0, stg_cutoff: float = 1.0):
    """_denoise_loop_cfg_av (av_pipeline.py:625-756) without gradient
    estimation or masks: ``model_fn(video_latent, audio_latent, sigma,
    pass_)`` -> (video velocity, audio velocity) for one batch row, pass_ in
    {"positive", "negative", "perturbed"}; the negative pass runs when either
    scale is not 1, the perturbed (STG) pass while stg_scale != 0 and
    (step + 1) / steps <= stg_cutoff (av_pipeline.py:706-717).  Returns the
    final (video, audio) latents."""
    need_cfg = cfg_video != 1.0 or cfg_audio != 1.0
    sig = np.asarray(sigmas, dtype=F32)
    steps = len(sig) - 1
    for i in range(steps):
        s, sn = float(sig[i]), float(sig[i + 1])
        vc, ac = model_fn(video_latent, audio_latent, s, "positive")
        vu = au = vp = None
        if need_cfg:
            vu, au = model_fn(video_latent, audio_latent, s, "negative")
        stg = stg_scale != 0.0 and (i + 1) / steps <= stg_cutoff
        if stg:
            vp, _ = model_fn(video_latent, audio_latent, s, "perturbed")
        video_latent = denoise_update(video_latent, vc, s, sn, v_uncond=vu, cfg_scale=cfg_video if need_cfg else 1.0,
                                      v_perturbed=vp, stg_scale=stg_scale if stg else 0.0)[0]
        audio_latent = denoise_update(audio_latent, ac, s, sn, v_uncond=au, cfg_scale=cfg_audio if need_cfg else 1.0)[0]
    return video_latent, audio_latent


def cfg_guide(cond, uncond, scale: float):
    """CFGGuider.guide (guiders.py:24-29), fp32."""
    c, u = np.asarray(cond, F32), np.asarray(uncond, F32)
    return (c + (F32(scale - 1) * (c - u).astype(F32)).astype(F32)).astype(F32)


def stg_guide(pos, perturbed, scale: float):
    """STGGuider.guide (guiders.py:79-83), fp32."""
    p, q = np.asarray(pos, F32), np.asarray(perturbed, F32)
    return (p + (F32(scale) * (p - q).astype(F32)).astype(F32)).astype(F32)


def cfg_star_guide(cond, uncond, scale: float):
    """CFGStarRescalingGuider.guide (guiders.py:35-62, projection_coef
    :174-192): the per-sample coefficient in float64, the rest fp32."""
    c, u = np.asarray(cond, F32), np.asarray(uncond, F32)
    b = c.shape[0]
    cf, uf = c.reshape(b, -1).astype(np.float64), u.reshape(b, -1).astype(np.float64)
    coef = ((cf * uf).sum(1) / ((uf * uf).sum(1) + 1e-8)).astype(F32).reshape((b,) + (1,) * (c.ndim - 1))
    return (c + (F32(scale - 1) * (c - (coef * u).astype(F32)).astype(F32)).astype(F32)).astype(F32)


def euler_step(sample, denoised, sigma: float, sigma_next: float):
    """EulerDiffusionStep.step (diffusion_steps.py:19-70) for a bf16 sample:
    bf16(d + fp32(sigma_next / sigma) (x - d))."""
    x, d = np.asarray(sample, F32), np.asarray(denoised, F32)
    r = F32(float(sigma_next) / float(sigma))
    return rbf16((d + (r * (x - d).astype(F32)).astype(F32)).astype(F32))


def heun_step(sample, denoised, sigma: float, sigma_next: float, denoised_at_predicted=None):
    """HeunDiffusionStep.step (diffusion_steps.py:72-130) for a bf16 sample,
    fp32 sigmas: Euler predictor; with the second prediction, the average of
    the two velocities."""
    x, d = np.asarray(sample, F32), np.asarray(denoised, F32)
    s, sn = F32(sigma), F32(sigma_next)
    dt = F32(sn - s)
    v1 = ((x - d).astype(F32) / s).astype(F32)
    pred = (x + (v1 * dt).astype(F32)).astype(F32)
    if denoised_at_predicted is None:
        return rbf16(pred)
    v2 = ((rbf16(pred) - np.asarray(denoised_at_predicted, F32)).astype(F32) / sn).astype(F32)
    avg = (F32(0.5) * (v1 + v2).astype(F32)).astype(F32)
    return rbf16((x + (avg * dt).astype(F32)).astype(F32))


def denoise_loop_av_general(model_fn, video_latent, audio_latent, sigmas, cfg_video: float = 1.0,
                            cfg_audio: float = 1.0, stg_scale: float = 0.0, stg_cutoff: float = 1.0,
                            ge_gamma: float = 0.0, video_mask=None, video_clean=None, audio_mask=None,
                            audio_clean=None):
    """_denoise_loop_cfg_av (av_pipeline.py:625-756) with every option:
    ``model_fn(video_latent, audio_latent, video_timesteps, audio_timesteps,
    pass_)`` -> velocities, timesteps fp32 (B,) or per token (B, T) (mask *
    sigma, pipelines/common.py:194-250); gradient estimation on the video
    stream; masks blend the clean latents back (common.py:169-191)."""
    need_cfg = cfg_video != 1.0 or cfg_audio != 1.0
    sig = np.asarray(sigmas, dtype=F32)
    steps = len(sig) - 1
    b = np.asarray(video_latent).shape[0]
    prev = None

    def ts(mask, s):
        full = np.full((b,), F32(s), F32)
        return full if mask is None else (np.asarray(mask, F32) * F32(s)).astype(F32)

    for i in range(steps):
        s, sn = float(sig[i]), float(sig[i + 1])
        vt, at = ts(video_mask, s), ts(audio_mask, s)
        vc, ac = model_fn(video_latent, audio_latent, vt, at, "positive")
        vu = au = vp = None
        if need_cfg:
            vu, au = model_fn(video_latent, audio_latent, vt, at, "negative")
        stg = stg_scale != 0.0 and (i + 1) / steps <= stg_cutoff
        if stg:
            vp, _ = model_fn(video_latent, audio_latent, vt, at, "perturbed")
        new_v, cur = denoise_update(video_latent, vc, s, sn, v_uncond=vu, cfg_scale=cfg_video if need_cfg else 1.0,
                                    v_perturbed=vp, stg_scale=stg_scale if stg else 0.0, denoise_mask=video_mask,
                                    clean_latent=video_clean, prev_velocity=prev, ge_gamma=ge_gamma)
        if ge_gamma > 0:
            prev = cur
        audio_latent = denoise_update(audio_latent, ac, s, sn, v_uncond=au, cfg_scale=cfg_audio if need_cfg else 1.0,
                                      denoise_mask=audio_mask, clean_latent=audio_clean)[0]
        video_latent = new_v
    return video_latent, audio_latent


def _post_process(d, mask, clean):
    """post_process_latent (common.py:169-191) in fp32."""
    if mask is None:
        return d
    m = np.asarray(mask, F32)[..., None]
    return ((d * m).astype(F32) + (np.asarray(clean, F32) * (F32(1.0) - m).astype(F32)).astype(F32)).astype(F32)


def denoise_loop_heun_av(model_fn, video_latent, audio_latent, sigmas, cfg_video: float = 1.0,
                         cfg_audio: float = 1.0, stg_scale: float = 0.0, stg_cutoff: float = 1.0,
                         ge_gamma: float = 0.0, video_mask=None, video_clean=None, audio_mask=None,
                         audio_clean=None):
    """_denoise_loop_heun_av (av_pipeline.py:758-897) with ``model_fn`` as
    in ``denoise_loop_av_general``: the guided X0 at the current point
    (CFG, STG, gradient estimation, mask blend), the Euler predictor, the
    guided X0 at the predicted point (CFG, mask blend) and the Heun
    corrector; at sigma_next = 0 the latent becomes the fp32 X0."""
    need_cfg = cfg_video != 1.0 or cfg_audio != 1.0
    sig = np.asarray(sigmas, dtype=F32)
    steps = len(sig) - 1
    b = np.asarray(video_latent).shape[0]
    prev = None

    def ts(mask, s):
        full = np.full((b,), F32(s), F32)
        return full if mask is None else (np.asarray(mask, F32) * F32(s)).astype(F32)

    def x0(lat, t, v):
        t = t[:, None, None] if t.ndim == 1 else t[:, :, None]
        return _x0(np.asarray(lat, F32), t, np.asarray(v, F32))

    def guided(vlat, alat, s):
        vt, at = ts(video_mask, s), ts(audio_mask, s)
        vc, ac = model_fn(vlat, alat, vt, at, "positive")
        dv, da = x0(vlat, vt, vc), x0(alat, at, ac)
        if need_cfg:
            vu, au = model_fn(vlat, alat, vt, at, "negative")
            dv, da = cfg_guide(dv, x0(vlat, vt, vu), cfg_video), cfg_guide(da, x0(alat, at, au), cfg_audio)
        return dv, da, vt

    for i in range(steps):
        s, sn = float(sig[i]), float(sig[i + 1])
        dv, da, vt = guided(video_latent, audio_latent, s)
        if stg_scale != 0.0 and (i + 1) / steps <= stg_cutoff:
            at = ts(audio_mask, s)
            vp, _ = model_fn(video_latent, audio_latent, vt, at, "perturbed")
            dv = stg_guide(dv, x0(video_latent, vt, vp), stg_scale)
        if ge_gamma > 0 and s > 0:
            x = np.asarray(video_latent, F32)
            cur = ((x - dv).astype(F32) / F32(s)).astype(F32)
            if prev is not None:
                total = ((F32(ge_gamma) * (cur - prev).astype(F32)).astype(F32) + prev).astype(F32)
                dv = (x - (total * F32(s)).astype(F32)).astype(F32)
            prev = cur
        dv, da = _post_process(dv, video_mask, video_clean), _post_process(da, audio_mask, audio_clean)
        if sn == 0:
            video_latent, audio_latent = dv, da
            continue
        dt = F32(F32(sn) - F32(s))
        pv = [rbf16((np.asarray(lat, F32) + (((np.asarray(lat, F32) - d).astype(F32) / F32(s)).astype(F32)
                                                 * dt).astype(F32)).astype(F32)) for lat, d in ((video_latent, dv),
                                                                                              (audio_latent, da))]
        dv2, da2, _ = guided(pv[0], pv[1], sn)
        dv2, da2 = _post_process(dv2, video_mask, video_clean), _post_process(da2, audio_mask, audio_clean)
        video_latent = heun_step(video_latent, dv, s, sn, dv2)
        audio_latent = heun_step(audio_latent, da, s, sn, da2)
    return video_latent, audio_latent
