"""GPU parity of the callers around the block loop: the fused denoise-step
kernel (bit-exact against the oracle's fp32 op sequence), the velocity model
(preprocess + blocks + output head) and the CFG-batched AV denoise loop
(within the block tolerance of the oracle; graph replay = eager)."""

import numpy as np
import pytest

from helpers import bf16_bits, block_params, from_dev_bf16, gpu_block, normal_bf16, normal_f32, rng, rope_np, \
    to_dev_bf16
from oracle import denoise as od
from oracle import ref_ops as ro
from oracle.bf16 import f32_to_bf16_bits

pytestmark = pytest.mark.gpu


def _f32_dev(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


@pytest.mark.parametrize("shape", [(2, 333, 128), (1, 77, 64), (3, 9, 8)])
@pytest.mark.parametrize("cfg,stg,mask,ge", [(1.0, 0.0, False, 0), (3.0, 0.0, False, 0), (4.5, 1.25, False, 0),
                                             (2.0, 0.0, True, 0), (1.0, 0.0, False, 1), (3.0, 0.5, True, 2)])
def test_denoise_update_matches_oracle_bitwise(cuda, shape, cfg, stg, mask, ge):
    """ge = 1: first step with gradient estimation (records the velocity),
    ge = 2: a later step (blends with the recorded one)."""
    import torch

    from ltxq.denoise import denoise_update

    g = rng(sum(shape) + int(cfg * 10) + ge)
    x, vc, vu, vp, clean = (normal_bf16(g, shape) for _ in range(5))
    m = (g.uniform(0, 1, shape[:2]) > 0.3).astype(np.float32) * g.uniform(0.5, 1, shape[:2]).astype(np.float32)
    prev = normal_f32(g, shape, 0.5)
    s, sn = 0.909375, 0.725
    ref, cur = od.denoise_update(x, vc, s, sn, v_uncond=vu, cfg_scale=cfg, v_perturbed=vp, stg_scale=stg,
                                 denoise_mask=m if mask else None, clean_latent=clean if mask else None,
                                 prev_velocity=prev if ge == 2 else None, ge_gamma=1.5 if ge else 0.0)
    prev_dev = _f32_dev(prev) if ge else None
    out = denoise_update(to_dev_bf16(x), to_dev_bf16(vc), s, sn, v_uncond=to_dev_bf16(vu), cfg_scale=cfg,
                         v_perturbed=to_dev_bf16(vp), stg_scale=stg, denoise_mask=_f32_dev(m) if mask else None,
                         clean_latent=to_dev_bf16(clean) if mask else None, prev_velocity=prev_dev,
                         ge_gamma=1.5 if ge else 0.0, have_prev=ge == 2)
    assert np.array_equal(bf16_bits(out), f32_to_bf16_bits(ref))
    if ge:
        assert np.array_equal(prev_dev.cpu().numpy().view(np.uint32), cur.view(np.uint32))
    assert torch.isfinite(out.float()).all()


def test_denoise_update_in_place_final_step_and_errors(cuda):
    import torch

    from ltxq.denoise import denoise_update

    g = rng(7)
    shape = (1, 256, 128)
    x, v, u = (normal_bf16(g, shape) for _ in range(3))
    for s, sn in ((1.0, 0.99375), (0.421875, 0.0)):  # sigma_next = 0: the last step returns the x0
        ref, _ = od.denoise_update(x, v, s, sn, v_uncond=u, cfg_scale=2.5)
        lat = to_dev_bf16(x)
        out = denoise_update(lat, to_dev_bf16(v), s, sn, v_uncond=to_dev_bf16(u), cfg_scale=2.5, out=lat)
        assert out.data_ptr() == lat.data_ptr()
        assert np.array_equal(bf16_bits(lat), f32_to_bf16_bits(ref))
    empty = torch.empty((0, 4, 8), dtype=torch.bfloat16, device="cuda")
    assert denoise_update(empty, empty, 0.5, 0.25).shape == (0, 4, 8)
    lat = to_dev_bf16(x)
    with pytest.raises(ValueError):
        denoise_update(lat, lat, 0.0, 0.0)  # sigma must be > 0
    with pytest.raises(ValueError):
        denoise_update(lat, lat, 0.5, 0.25, cfg_scale=3.0)  # CFG without the negative velocity
    with pytest.raises(ValueError):
        denoise_update(lat, lat[:, :128], 0.5, 0.25)


VIDEO = (1024, 8, 128, 1024)
AUDIO = (512, 8, 64, 512)


def _model_case(n_blocks=2, seed=40):
    """Random small model: GPU ``LTXAVModel`` and the oracle's parameters."""
    import torch

    from ltxq.block import StreamConfig
    from ltxq.model import LTXAVModel, model_param_specs

    video, audio = StreamConfig(*VIDEO), StreamConfig(*AUDIO)
    blocks, blocks_p = [], []
    for i in range(n_blocks):
        p_oracle, quant, tables = block_params(video, audio, "mxfp8", 8, seed=seed + i)
        blocks_p.append(p_oracle)
        blocks.append(gpu_block(quant, tables, video, audio, "mxfp8"))
    g = rng(seed + 100)
    mp, state = {}, {}
    for key, shape in model_param_specs(video, audio).items():
        if key.endswith("scale_shift_table"):
            a = normal_f32(g, shape, 0.1)
            state[key] = torch.from_numpy(a).cuda()
        else:
            a = normal_bf16(g, shape, 0.01 if key.endswith(".bias") else 0.02)
            state[key] = to_dev_bf16(a)
        mp[key] = a
    return LTXAVModel.from_state(blocks, state, video, audio), blocks_p, mp, video, audio


def _stream_inputs(g, cfg, tokens, ctx_tokens, cross_heads, cross_d):
    return {"latent": normal_bf16(g, (tokens, 128)), "context": normal_bf16(g, (ctx_tokens, cfg.context_dim)),
            "pe": rope_np(g, cfg.heads, tokens, cfg.d_head), "cross_pe": rope_np(g, cross_heads, tokens, cross_d)}


def _pe_dev(pe, batch=1):
    import torch

    return tuple(torch.stack([_f32_dev(c)] * batch) for c in pe)


def test_model_matches_oracle(cuda):
    """LTXModel.__call__: preprocess (patchify, four AdaLN MLPs per stream),
    two blocks, output heads; velocities of both streams against the oracle
    at the block tolerance."""
    import torch

    import ltxq
    from ltxq.model import Modality

    model, blocks_p, mp, video, audio = _model_case()
    g = rng(41)
    T, A, L = 64, 32, 24
    vs = _stream_inputs(g, video, T, L, audio.heads, audio.d_head)
    as_ = _stream_inputs(g, audio, A, L, audio.heads, audio.d_head)
    sigma = 0.909375
    ref_v, ref_a = od.model_forward(blocks_p, mp, dict(vs, sigma=sigma), dict(as_, sigma=sigma), video.heads,
                                    audio.heads)
    sig = torch.full((1,), sigma, dtype=torch.float32, device="cuda")
    vm = Modality(to_dev_bf16(vs["latent"])[None], sig, to_dev_bf16(vs["context"])[None], _pe_dev(vs["pe"]),
                  _pe_dev(vs["cross_pe"]), sigma=sig)
    am = Modality(to_dev_bf16(as_["latent"])[None], sig, to_dev_bf16(as_["context"])[None], _pe_dev(as_["pe"]),
                  _pe_dev(as_["cross_pe"]), sigma=sig)
    ov, oa = model(vm, am)
    assert ov.shape == (1, T, 128) and oa.shape == (1, A, 128) and ov.dtype == torch.bfloat16
    for got, ref, what in ((from_dev_bf16(ov[0]), ref_v, "video"), (from_dev_bf16(oa[0]), ref_a, "audio")):
        mar, cos = ro.max_abs_rel(got, ref), ro.cosine(got, ref)
        assert mar <= 2e-2 and cos >= 0.9995, f"{what}: max_abs_rel={mar:.3e} cos={cos:.6f}"
    assert ltxq._lib.device_error() == 0


def test_model_per_token_timesteps_matches_oracle(cuda):
    """A non-uniform denoise mask (conditioning tokens at mask 0): per-token
    video timesteps (mask * sigma) run the AdaLN MLPs per token and give
    per-token AdaLN vectors in every block and in the output head."""
    import torch

    import ltxq
    from ltxq.model import Modality

    model, blocks_p, mp, video, audio = _model_case(seed=60)
    g = rng(61)
    T, A, L = 64, 32, 24
    vs = _stream_inputs(g, video, T, L, audio.heads, audio.d_head)
    as_ = _stream_inputs(g, audio, A, L, audio.heads, audio.d_head)
    sigma = 0.725
    mask = np.ones(T, np.float32)
    mask[:16] = 0.0
    mask[16:24] = 0.5
    ts = (mask * np.float32(sigma)).astype(np.float32)
    ref_v, ref_a = od.model_forward(blocks_p, mp, dict(vs, sigma=sigma, timesteps=ts), dict(as_, sigma=sigma),
                                    video.heads, audio.heads)
    sig = torch.full((1,), sigma, dtype=torch.float32, device="cuda")
    vm = Modality(to_dev_bf16(vs["latent"])[None], _f32_dev(ts)[None], to_dev_bf16(vs["context"])[None],
                  _pe_dev(vs["pe"]), _pe_dev(vs["cross_pe"]), sigma=sig)
    am = Modality(to_dev_bf16(as_["latent"])[None], sig, to_dev_bf16(as_["context"])[None], _pe_dev(as_["pe"]),
                  _pe_dev(as_["cross_pe"]), sigma=sig)
    ov, oa = model(vm, am)
    for got, ref, what in ((from_dev_bf16(ov[0]), ref_v, "video"), (from_dev_bf16(oa[0]), ref_a, "audio")):
        mar, cos = ro.max_abs_rel(got, ref), ro.cosine(got, ref)
        assert mar <= 2e-2 and cos >= 0.9995, f"{what}: max_abs_rel={mar:.3e} cos={cos:.6f}"
    assert ltxq._lib.device_error() == 0


def test_denoise_loop_cfg_matches_oracle_and_graph_replay(cuda):
    """Two steps of the AV CFG loop (positive and negative passes batched
    into one batch-2 transformer pass) against the oracle loop, which runs
    the two passes separately; the CUDA-graph loop matches the eager one."""
    import torch

    import ltxq
    from ltxq.denoise import CFGGuider, LatentState, denoise_av

    model, blocks_p, mp, video, audio = _model_case(seed=50)
    g = rng(51)
    T, A, L = 64, 32, 24
    vs = _stream_inputs(g, video, T, L, audio.heads, audio.d_head)
    as_ = _stream_inputs(g, audio, A, L, audio.heads, audio.d_head)
    neg_v = normal_bf16(g, (L, video.context_dim))
    neg_a = normal_bf16(g, (L, audio.context_dim))
    sigmas = np.asarray([1.0, 0.909375, 0.725], np.float32)
    cfg_v, cfg_a = 2.0, 1.5

    def oracle_model(vl, al, s, pass_):
        negative = pass_ == "negative"
        v_in = dict(vs, latent=vl, sigma=s, context=neg_v if negative else vs["context"])
        a_in = dict(as_, latent=al, sigma=s, context=neg_a if negative else as_["context"])
        return od.model_forward(blocks_p, mp, v_in, a_in, video.heads, audio.heads)

    ref_v, ref_a = od.denoise_loop_av(oracle_model, vs["latent"], as_["latent"], sigmas, cfg_v, cfg_a)

    outs = []
    for graph in (False, True):
        vst = LatentState(to_dev_bf16(vs["latent"])[None])
        ast = LatentState(to_dev_bf16(as_["latent"])[None])
        fv, fa = denoise_av(model, vst, ast, sigmas, to_dev_bf16(vs["context"])[None],
                            to_dev_bf16(as_["context"])[None], _pe_dev(vs["pe"]), _pe_dev(as_["pe"]),
                            _pe_dev(vs["cross_pe"]), _pe_dev(as_["cross_pe"]),
                            negative_video_context=to_dev_bf16(neg_v)[None],
                            negative_audio_context=to_dev_bf16(neg_a)[None], video_guider=CFGGuider(cfg_v),
                            audio_guider=CFGGuider(cfg_a), graph=graph)
        outs.append((fv.latent.clone(), fa.latent.clone()))
    for a, b in zip(outs[0], outs[1]):  # graph vs eager: same kernels (cuBLAS may pick another fp32 algorithm)
        assert ro.max_abs_rel(from_dev_bf16(b), from_dev_bf16(a)) <= 2e-3
    for got, ref, what in ((from_dev_bf16(outs[0][0][0]), ref_v, "video"),
                           (from_dev_bf16(outs[0][1][0]), ref_a, "audio")):
        mar, cos = ro.max_abs_rel(got, ref), ro.cosine(got, ref)
        assert mar <= 2e-2 and cos >= 0.9995, f"{what}: max_abs_rel={mar:.3e} cos={cos:.6f}"
    assert ltxq._lib.device_error() == 0


SKIPS = {0: frozenset({"skip_video_self_attn", "skip_audio_self_attn"}),
         1: frozenset({"skip_a2v_cross_attn", "skip_v2a_cross_attn"})}


def _perturbations(batch):
    from ltxq.perturbations import BatchedPerturbationConfig, Perturbation, PerturbationConfig, PerturbationType

    cfg = PerturbationConfig([Perturbation(PerturbationType.SKIP_VIDEO_SELF_ATTN, [0]),
                              Perturbation(PerturbationType.SKIP_AUDIO_SELF_ATTN, [0]),
                              Perturbation(PerturbationType.SKIP_A2V_CROSS_ATTN, [1]),
                              Perturbation(PerturbationType.SKIP_V2A_CROSS_ATTN, [1])])
    return BatchedPerturbationConfig([cfg] * batch)


def test_model_perturbed_pass_matches_oracle(cuda):
    """The STG perturbed pass: block 0 skips both self-attentions, block 1
    both audio<->video cross-attentions; against the oracle with the same
    skips."""
    import torch

    import ltxq
    from ltxq.model import Modality

    model, blocks_p, mp, video, audio = _model_case(seed=70)
    g = rng(71)
    T, A, L = 64, 32, 24
    vs = _stream_inputs(g, video, T, L, audio.heads, audio.d_head)
    as_ = _stream_inputs(g, audio, A, L, audio.heads, audio.d_head)
    sigma = 0.98125
    ref_v, ref_a = od.model_forward(blocks_p, mp, dict(vs, sigma=sigma), dict(as_, sigma=sigma), video.heads,
                                    audio.heads, skips=SKIPS)
    sig = torch.full((1,), sigma, dtype=torch.float32, device="cuda")
    vm = Modality(to_dev_bf16(vs["latent"])[None], sig, to_dev_bf16(vs["context"])[None], _pe_dev(vs["pe"]),
                  _pe_dev(vs["cross_pe"]), sigma=sig)
    am = Modality(to_dev_bf16(as_["latent"])[None], sig, to_dev_bf16(as_["context"])[None], _pe_dev(as_["pe"]),
                  _pe_dev(as_["cross_pe"]), sigma=sig)
    ov, oa = model(vm, am, perturbations=_perturbations(1))
    full_v, _ = model(vm, am)
    for got, ref, what in ((from_dev_bf16(ov[0]), ref_v, "video"), (from_dev_bf16(oa[0]), ref_a, "audio")):
        mar, cos = ro.max_abs_rel(got, ref), ro.cosine(got, ref)
        assert mar <= 2e-2 and cos >= 0.9995, f"{what}: max_abs_rel={mar:.3e} cos={cos:.6f}"
    assert not torch.equal(full_v.view(torch.int16), ov.view(torch.int16))  # the skips change the result
    assert ltxq._lib.device_error() == 0


def test_denoise_loop_stg_matches_oracle(cuda):
    """Two steps of the loop with CFG and STG (the perturbed pass in the
    first step only: cutoff 0.5) against the oracle loop, eager and with
    both passes replayed as CUDA graphs."""
    import ltxq
    from ltxq.denoise import CFGGuider, LatentState, STGGuider, denoise_av

    model, blocks_p, mp, video, audio = _model_case(seed=80)
    g = rng(81)
    T, A, L = 64, 32, 24
    vs = _stream_inputs(g, video, T, L, audio.heads, audio.d_head)
    as_ = _stream_inputs(g, audio, A, L, audio.heads, audio.d_head)
    neg_v = normal_bf16(g, (L, video.context_dim))
    neg_a = normal_bf16(g, (L, audio.context_dim))
    sigmas = np.asarray([1.0, 0.909375, 0.725], np.float32)

    def oracle_model(vl, al, s, pass_):
        negative = pass_ == "negative"
        v_in = dict(vs, latent=vl, sigma=s, context=neg_v if negative else vs["context"])
        a_in = dict(as_, latent=al, sigma=s, context=neg_a if negative else as_["context"])
        return od.model_forward(blocks_p, mp, v_in, a_in, video.heads, audio.heads,
                                skips=SKIPS if pass_ == "perturbed" else None)

    ref_v, ref_a = od.denoise_loop_av(oracle_model, vs["latent"], as_["latent"], sigmas, 2.0, 1.5, stg_scale=1.0,
                                      stg_cutoff=0.5)
    outs = []
    for graph in (False, True):
        fv, fa = denoise_av(model, LatentState(to_dev_bf16(vs["latent"])[None]),
                            LatentState(to_dev_bf16(as_["latent"])[None]), sigmas, to_dev_bf16(vs["context"])[None],
                            to_dev_bf16(as_["context"])[None], _pe_dev(vs["pe"]), _pe_dev(as_["pe"]),
                            _pe_dev(vs["cross_pe"]), _pe_dev(as_["cross_pe"]),
                            negative_video_context=to_dev_bf16(neg_v)[None],
                            negative_audio_context=to_dev_bf16(neg_a)[None], video_guider=CFGGuider(2.0),
                            audio_guider=CFGGuider(1.5), stg_guider=STGGuider(1.0), stg_perturbations=_perturbations(1),
                            stg_cutoff=0.5, graph=graph)
        outs.append((from_dev_bf16(fv.latent[0]), from_dev_bf16(fa.latent[0])))
    for got, ref, what in ((outs[0][0], ref_v, "video"), (outs[0][1], ref_a, "audio")):
        mar, cos = ro.max_abs_rel(got, ref), ro.cosine(got, ref)
        assert mar <= 2e-2 and cos >= 0.9995, f"{what}: max_abs_rel={mar:.3e} cos={cos:.6f}"
    for a, b in zip(outs[0], outs[1]):
        assert ro.max_abs_rel(b, a) <= 2e-3
    assert ltxq._lib.device_error() == 0
