"""GPU: blocks loaded from a cache on disk (the reference's key scheme,
shards, metadata.json) compute the same bits as the blocks they were written
from."""

import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode,bits,payload_mode", [("mxfp8", 8, "mxfp8-blocks"), ("affine", 8, "off"),
                                                   ("mxfp8", 8, "mxfp8-blocks-pretranspose")])
def test_blocks_from_cache_match_source(cuda, tmp_path, mode, bits, payload_mode):
    import torch

    import ltxq
    from ltxq import cache as C
    from ltxq.block import BasicAVTransformerBlock, StreamConfig, TransformerArgs

    pt = payload_mode == "mxfp8-blocks-pretranspose"
    # pretransposed groups run along the output dimension, so every output
    # width (the per-head gate logits included) is a multiple of 32
    video = StreamConfig(2048, 32, 64, 2048) if pt else StreamConfig(1024, 8, 128, 1024)
    audio = StreamConfig(2048, 32, 64, 2048) if pt else StreamConfig(512, 8, 64, 512)
    T, A, L = 80, 40, 24
    gen = torch.Generator(device="cuda")
    gen.manual_seed(11)
    parts = [BasicAVTransformerBlock.random_parts(gen, "cuda", mode=mode, bits=bits, video=video, audio=audio,
                                                  pretransposed=pt) for _ in range(2)]
    state = {}
    for i, (lin, tabs) in enumerate(parts):
        state.update(C.block_state(i, lin, tabs))
    cache_file = tmp_path / "transformer.safetensors"
    shards = C.write_cache_weights(cache_file, state, shard_limit_bytes=8 << 20)
    assert len(shards) > 1
    extra = {"video_ff_quantize_bits": bits} if mode == "affine" else {}
    C.write_metadata(tmp_path, C.cache_payload(payload_mode, **extra))
    loaded = C.blocks_from_cache(cache_file, "cuda", video, audio)
    direct = [BasicAVTransformerBlock(lin, tabs, video, audio) for lin, tabs in parts]
    assert len(loaded) == 2

    def rnd(*shape, std=1.0, dtype=torch.float32):
        return (torch.randn(*shape, generator=gen, device="cuda") * std).to(dtype)

    def rope(heads, t, d):
        ang = torch.rand(1, heads, t, d // 2, generator=gen, device="cuda") * 6.28
        return torch.cos(ang), torch.sin(ang)

    def args(cfg, t):
        return TransformerArgs(x=rnd(1, t, cfg.dim, dtype=torch.bfloat16),
                               context=rnd(1, L, cfg.context_dim, dtype=torch.bfloat16),
                               timesteps=rnd(1, 1, 9, cfg.dim, std=0.1),
                               positional_embeddings=rope(cfg.heads, t, cfg.d_head),
                               cross_positional_embeddings=rope(audio.heads, t, audio.d_head),
                               cross_scale_shift_timestep=rnd(1, 1, 4, cfg.dim, std=0.1),
                               cross_gate_timestep=rnd(1, 1, 1, cfg.dim, std=0.1),
                               prompt_timestep=rnd(1, 1, 2, cfg.dim, std=0.1))

    v, a = args(video, T), args(audio, A)
    outs = []
    for blocks in (direct, loaded):
        vv, aa = v, a
        for b in blocks:
            vv, aa = b(vv, aa)
        outs.append((vv.x.clone(), aa.x.clone()))
    assert torch.equal(outs[0][0].view(torch.int16), outs[1][0].view(torch.int16))
    assert torch.equal(outs[0][1].view(torch.int16), outs[1][1].view(torch.int16))
    assert ltxq._lib.device_error() == 0


def _to_checkpoint_key(base: str) -> str:
    """MLX base name -> the checkpoint's PyTorch name (inverse of the
    reference's weight_converter renames)."""
    for mlx, pt in (("audio_ff.project_in.proj", "audio_ff.net.0.proj"), ("audio_ff.project_out", "audio_ff.net.2"),
                    ("ff.project_in.proj", "ff.net.0.proj"), ("ff.project_out", "ff.net.2")):
        if base == mlx:
            return pt
    return base.replace(".to_out", ".to_out.0")


@pytest.mark.parametrize("mode,affine", [("mxfp8-blocks", None), ("off", (8, 64))])
def test_cache_built_from_checkpoint_matches_direct_blocks(cuda, tmp_path, mode, affine):
    """A bf16 checkpoint with the reference's PyTorch key names, built into a
    cache (quantized on the GPU) and loaded back, gives the same block output
    bits as blocks quantized directly from the same weights."""
    import torch

    from ltxq import cache as C
    from ltxq import cache_build as CB
    from ltxq.block import BasicAVTransformerBlock, StreamConfig, TransformerArgs, linear_specs, table_specs
    from ltxq.quantized_linear import QuantizedLinear

    video = StreamConfig(1024, 8, 128, 1024)
    audio = StreamConfig(512, 8, 64, 512)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(21)
    ckpt, direct = {}, []
    for i in range(2):
        lin, tabs = {}, {}
        for base, (n, k) in linear_specs(video, audio).items():
            w = (torch.randn(n, k, generator=gen, device="cuda") * 0.02).to(torch.bfloat16)
            b = (torch.randn(n, generator=gen, device="cuda") * 0.01).to(torch.bfloat16)
            pk = f"model.diffusion_model.transformer_blocks.{i}.{_to_checkpoint_key(base)}"
            ckpt[f"{pk}.weight"], ckpt[f"{pk}.bias"] = w, b
            lin[base] = (QuantizedLinear.from_linear(w, b, group_size=affine[1], bits=affine[0], mode="affine")
                         if affine else QuantizedLinear.from_linear(w, b, mode="mxfp8"))
        for name, shape in table_specs(video, audio).items():
            t = torch.randn(*shape, generator=gen, device="cuda") * 0.1
            t = (1.0 + t) if name.endswith("norm.weight") else t
            ckpt[f"model.diffusion_model.transformer_blocks.{i}.{name}"] = t
            tabs[name] = t
        direct.append(BasicAVTransformerBlock(lin, tabs, video, audio))
    ck = tmp_path / "ckpt.safetensors"
    C.save_safetensors(ck, ckpt)
    cache_file = tmp_path / "cache" / "transformer.safetensors"
    CB.build_transformer_cache(ck, cache_file, mode=mode, affine=affine, shard_limit_bytes=8 << 20)
    loaded = C.blocks_from_cache(cache_file, "cuda", video, audio)

    def rnd(*shape, std=1.0, dtype=torch.float32):
        return (torch.randn(*shape, generator=gen, device="cuda") * std).to(dtype)

    def rope(heads, t, d):
        ang = torch.rand(1, heads, t, d // 2, generator=gen, device="cuda") * 6.28
        return torch.cos(ang), torch.sin(ang)

    def args(cfg, t):
        return TransformerArgs(x=rnd(1, t, cfg.dim, dtype=torch.bfloat16), context=rnd(1, 24, cfg.context_dim,
                                                                                         dtype=torch.bfloat16),
                               timesteps=rnd(1, 1, 9, cfg.dim, std=0.1),
                               positional_embeddings=rope(cfg.heads, t, cfg.d_head),
                               cross_positional_embeddings=rope(audio.heads, t, audio.d_head),
                               cross_scale_shift_timestep=rnd(1, 1, 4, cfg.dim, std=0.1),
                               cross_gate_timestep=rnd(1, 1, 1, cfg.dim, std=0.1),
                               prompt_timestep=rnd(1, 1, 2, cfg.dim, std=0.1))

    v, a = args(video, 64), args(audio, 32)
    outs = []
    for blocks in (direct, loaded):
        vv, aa = v, a
        for blk in blocks:
            vv, aa = blk(vv, aa)
        outs.append((vv.x.clone(), aa.x.clone()))
    assert torch.equal(outs[0][0].view(torch.int16), outs[1][0].view(torch.int16))
    assert torch.equal(outs[0][1].view(torch.int16), outs[1][1].view(torch.int16))
