"""CPU tests of the model wrapper's host side: the non-block parameter names
(the reference's keys, model/transformer/model.py:640-712), their round
trip through the cache format, and the torch composition of the timestep
embedding and AdaLN MLP (timestep_embedding.py:8-201) against the oracle.
These pieces compute nothing on the library's CUDA path; the GPU tests cover
the model end to end."""

import numpy as np
import pytest
import torch

from oracle import denoise as od


def test_non_block_parameter_names_and_shapes():
    from ltxq.model import model_param_specs

    specs = model_param_specs()
    # spot checks against the reference's module tree for the 22B model
    assert specs["patchify_proj.weight"] == (4096, 128)
    assert specs["audio_patchify_proj.weight"] == (2048, 128)
    assert specs["adaln_single.emb.timestep_embedder.linear_1.weight"] == (4096, 256)
    assert specs["adaln_single.linear.weight"] == (9 * 4096, 4096)
    assert specs["prompt_adaln_single.linear.weight"] == (2 * 4096, 4096)
    assert specs["audio_prompt_adaln_single.linear.weight"] == (2 * 2048, 2048)
    assert specs["av_ca_video_scale_shift_adaln_single.linear.weight"] == (4 * 4096, 4096)
    assert specs["av_ca_a2v_gate_adaln_single.linear.weight"] == (4096, 4096)
    assert specs["av_ca_audio_scale_shift_adaln_single.linear.weight"] == (4 * 2048, 2048)
    assert specs["av_ca_v2a_gate_adaln_single.linear.weight"] == (2048, 2048)
    assert specs["scale_shift_table"] == (2, 4096) and specs["audio_scale_shift_table"] == (2, 2048)
    assert specs["proj_out.weight"] == (128, 4096) and specs["audio_proj_out.bias"] == (128,)
    assert not any(k.startswith("transformer_blocks.") for k in specs)
    assert set(od.MODEL_PREFIXES["video"].values()) | set(od.MODEL_PREFIXES["audio"].values()) == {
        k.split(".")[0] for k in specs}


def test_model_state_round_trips_through_the_cache(tmp_path):
    from ltxq import cache as C
    from ltxq.block import StreamConfig
    from ltxq.model import _stream_from_state, model_param_specs, random_model_state

    video, audio = StreamConfig(256, 4, 64, 256), StreamConfig(128, 4, 32, 128)
    g = torch.Generator()
    g.manual_seed(3)
    state = random_model_state(g, "cpu", video, audio)
    assert set(state) == set(model_param_specs(video, audio))
    C.write_cache_weights(tmp_path / "transformer.safetensors", state, shard_limit_bytes=1 << 20)
    back = C.load_cache_weights(tmp_path / "transformer.safetensors")
    assert set(back) == set(state)
    for k, t in state.items():
        assert back[k].dtype == t.dtype and torch.equal(back[k], t)
    s = _stream_from_state(back, "audio", audio)
    assert s.adaln.w.dtype == torch.float32 and s.adaln.w.shape == (9 * 128, 128) and s.adaln.n == 9
    assert s.cross_gate_adaln.w.shape == (128, 128) and s.prompt_adaln.n == 2
    assert s.patchify_w.dtype == torch.bfloat16 and s.proj_out_w.shape == (128, 128)
    assert s.scale_shift_table.dtype == torch.float32 and torch.equal(s.scale_shift_table,
                                                                      state["audio_scale_shift_table"])


@pytest.mark.parametrize("t", [[0.0], [1000.0], [909.375, 421.875, 1.0]])
def test_timestep_embedding_and_adaln_mlp_match_the_oracle(t):
    from ltxq.model import AdaLNSingle, timestep_embedding

    ts = torch.tensor(t, dtype=torch.float32)
    emb = timestep_embedding(ts).numpy()
    ref = od.timestep_embedding(np.asarray(t, np.float32))
    assert emb.shape == ref.shape == (len(t), 256)
    assert np.max(np.abs(emb - ref)) <= 1e-4  # fp32 sin/cos of arguments up to 1000 rad
    g = np.random.default_rng(5)
    d = 64
    p = {"linear_1.weight": g.standard_normal((d, 256)) * 0.02, "linear_1.bias": g.standard_normal(d) * 0.01,
         "linear_2.weight": g.standard_normal((d, d)) * 0.02, "linear_2.bias": g.standard_normal(d) * 0.01,
         "linear.weight": g.standard_normal((3 * d, d)) * 0.02, "linear.bias": g.standard_normal(3 * d) * 0.01}
    p = {k: v.astype(np.float32) for k, v in p.items()}
    state = {f"a.{'emb.timestep_embedder.' if k.startswith('linear_') else ''}{k}": torch.from_numpy(v)
             for k, v in p.items()}
    out, emb_t = AdaLNSingle.from_state(state, "a", 3)(ts)
    ref_out, ref_t = od.ada_single(p, np.asarray(t, np.float32))
    assert np.allclose(out.numpy(), ref_out, rtol=1e-4, atol=1e-5)
    assert np.allclose(emb_t.numpy(), ref_t, rtol=1e-4, atol=1e-5)


def test_v2_architecture_structure():
    """The LTX-2.3 (V2) structure the reference's tests/test_v2_architecture.py
    pins: 9-row AdaLN tables (6 base + 3 for the text cross-attention query),
    2-row prompt tables for the context K/V modulation, a per-head gate
    projection in every attention module, and no caption projection in the
    model."""
    from ltxq.block import AUDIO_22B, VIDEO_22B, attention_dims, linear_specs, table_specs
    from ltxq.cache import QUANTIZED_BLOCK_LINEAR_BASES
    from ltxq.model import model_param_specs

    tabs = table_specs()
    assert tabs["scale_shift_table"] == (9, VIDEO_22B.dim) and tabs["audio_scale_shift_table"] == (9, AUDIO_22B.dim)
    assert tabs["prompt_scale_shift_table"] == (2, VIDEO_22B.dim)
    assert tabs["scale_shift_table_a2v_ca_video"] == (5, VIDEO_22B.dim)
    lin = linear_specs()
    for name in ("attn1", "attn2", "audio_attn1", "audio_attn2", "audio_to_video_attn", "video_to_audio_attn"):
        qd, _, heads, _ = attention_dims(name, VIDEO_22B, AUDIO_22B)
        assert lin[f"{name}.to_gate_logits"] == (heads, qd)
    assert sorted(lin) == sorted(QUANTIZED_BLOCK_LINEAR_BASES) and len(lin) == 34
    assert not any("caption_projection" in k for k in model_param_specs())


def test_model_rope_tables_from_positions():
    """LTXAVModel builds the four RoPE tables of a stage from the token
    bounds as the reference's preprocessors do: video (dim 4096, 32 heads,
    max_pos (20, 2048, 2048)), audio and both cross tables (audio width and
    heads, max_pos (20,), temporal bounds only)."""
    from oracle import rope as orope

    from ltxq.block import StreamConfig
    from ltxq.model import LTXAVModel, random_model_state
    from ltxq.rope import audio_positions, video_positions

    video, audio = StreamConfig(256, 4, 64, 256), StreamConfig(128, 4, 32, 128)
    g = torch.Generator()
    g.manual_seed(4)
    model = LTXAVModel.from_state([], random_model_state(g, "cpu", video, audio), video, audio,
                                  use_double_precision_rope=True)
    vpos, apos = video_positions(1, 2, 3, 4, 24.0), audio_positions(1, 9)
    (vc, vs), (ac, as_), (vcc, vcs), (acc, acs) = model.positional_tables(vpos, apos)
    refs = [orope.precompute_freqs_cis(vpos.numpy(), 256, 10000.0, [20, 2048, 2048], True, 4, True),
            orope.precompute_freqs_cis(apos.numpy(), 128, 10000.0, [20], True, 4, True),
            orope.precompute_freqs_cis(vpos[:, 0:1].numpy(), 128, 10000.0, [20], True, 4, True),
            orope.precompute_freqs_cis(apos.numpy(), 128, 10000.0, [20], True, 4, True)]
    for (c, s), (rc, rs) in zip(((vc, vs), (ac, as_), (vcc, vcs), (acc, acs)), refs):
        assert c.shape == rc.shape
        assert np.max(np.abs(c.numpy() - rc)) <= 1e-6 and np.max(np.abs(s.numpy() - rs)) <= 1e-6
    assert vc.shape == (1, 4, 24, 32) and vcc.shape == (1, 4, 24, 16) and ac.shape == (1, 4, 9, 16)


def test_x0_model_matches_the_oracle_x0():
    """X0Model.denoise: bf16 latent - fp32 timesteps * bf16 velocity in fp32,
    uniform (B,) and per-token (B, T) timesteps."""
    from helpers import normal_bf16, rng
    from ltxq.model import Modality, X0Model

    g = rng(9)
    lat, vel = normal_bf16(g, (2, 6, 8)), normal_bf16(g, (2, 6, 8))
    to_t = lambda a: torch.from_numpy(a).to(torch.bfloat16)  # noqa: E731
    calls = []

    def velocity_model(video, audio, shard, perturbations):
        calls.append(perturbations)
        return to_t(vel), to_t(vel)

    x0 = X0Model(velocity_model)
    for ts in (np.array([0.725, 0.5], np.float32), np.array([[0.725] * 6, [0.0] * 3 + [0.5] * 3], np.float32)):
        m = Modality(to_t(lat), torch.from_numpy(ts), None)
        dv, da = x0(m, m, perturbations="ptb")
        t = ts[:, None, None] if ts.ndim == 1 else ts[:, :, None]
        ref = (lat - (t * vel).astype(np.float32)).astype(np.float32)
        assert dv.dtype == torch.float32 and np.array_equal(dv.numpy(), ref) and np.array_equal(da.numpy(), ref)
    assert calls == ["ptb", "ptb"]


def test_adaln_table_sums_in_one_multi_tensor_add():
    """BasicAVTransformerBlock._ada_prepare: every table + timestep sum of a
    block call from one torch._foreach_add equals the per-table broadcast
    add bit for bit (batch 2), and per-token timestep rows are left to the
    broadcast add."""
    import torch

    from ltxq.block import AUDIO_22B, VIDEO_22B, BasicAVTransformerBlock, TransformerArgs, table_specs

    g = torch.Generator().manual_seed(3)
    blk = object.__new__(BasicAVTransformerBlock)  # tables only: no quantized linears (they need a GPU)
    blk.tables = {k: torch.randn(*s, generator=g) * 0.1 for k, s in table_specs(VIDEO_22B, AUDIO_22B).items()}
    blk._expanded = {}

    def args(C, per_token=False):
        r = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
        return TransformerArgs(x=None, context=None, timesteps=r(2, 5 if per_token else 1, 9, C),
                               positional_embeddings=None, cross_positional_embeddings=None,
                               cross_scale_shift_timestep=r(2, 1, 4, C), cross_gate_timestep=r(2, 1, 1, C),
                               prompt_timestep=r(2, 1, 2, C))

    for per_token in (False, True):
        video, audio = args(VIDEO_22B.dim, per_token), args(AUDIO_22B.dim)
        blk._ada_rows = {}
        blk._ada_prepare(video, audio)
        assert (("scale_shift_table", id(video.timesteps)) in blk._ada_rows) == (not per_token)
        for tab, a in (("scale_shift_table", video), ("audio_scale_shift_table", audio)):
            got = blk._ada(tab, a.timesteps, 0, 9)
            ref = blk.tables[tab][None, None] + a.timesteps
            assert all(torch.equal(got[i], ref[:, :, i]) for i in range(9))
        for tab, a in (("scale_shift_table_a2v_ca_video", video), ("scale_shift_table_a2v_ca_audio", audio)):
            got = blk._ada_cross(tab, a)
            ref = blk.tables[tab][:4][None, None] + a.cross_scale_shift_timestep
            assert all(torch.equal(got[i], ref[:, :, i]) for i in range(4))
            assert torch.equal(blk._cross_gate(tab, a),
                               blk.tables[tab][4][None, None] + a.cross_gate_timestep[:, :, 0])
        for tab, a in (("prompt_scale_shift_table", video), ("audio_prompt_scale_shift_table", audio)):
            assert torch.equal(blk._ada_rows[(tab, id(a.prompt_timestep))],
                               blk.tables[tab][None, None] + a.prompt_timestep)
    # a table replaced by another tensor, or changed in place, is expanded again
    video, audio = args(VIDEO_22B.dim), args(AUDIO_22B.dim)
    for change in ("replace", "in_place"):
        if change == "replace":
            blk.tables["scale_shift_table"] = torch.randn(9, VIDEO_22B.dim, generator=g)
        else:
            blk.tables["scale_shift_table"].add_(1.0)
        blk._ada_rows = {}
        blk._ada_prepare(video, audio)
        got = blk._ada("scale_shift_table", video.timesteps, 0, 9)
        ref = blk.tables["scale_shift_table"][None, None] + video.timesteps
        assert all(torch.equal(got[i], ref[:, :, i]) for i in range(9)), change
