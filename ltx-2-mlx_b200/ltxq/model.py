"""The velocity model around the block loop: LTXModel of
LTX_2_MLX/model/transformer/model.py:454-1487 (AudioVideo, LTX-2.3).

One call is the reference's ``LTXModel.__call__`` (model.py:1344-1487):

* preprocess each stream (``TransformerArgsPreprocessor.prepare``
  model.py:285-340 and ``MultiModalTransformerArgsPreprocessor.prepare``
  :445-505): ``patchify_proj`` on the latent; the AdaLN MLPs
  (``AdaLayerNormSingle``, timestep_embedding.py:165-201) on timesteps x 1000
  (9 rows), on sigma x 1000 for the prompt K/V modulation (2 rows), on the
  stream's own timesteps x 1000 for the cross-attention scale/shift (4 rows,
  the "official" mode) and on the other stream's sigma x
  ``av_ca_timestep_scale_multiplier`` for the cross-attention gate (1 row);
* the 48 ``BasicAVTransformerBlock`` calls (``ltxq.block``);
* the output head (``_process_video_output`` / ``_process_audio_output``
  model.py:1312-1340): LayerNorm without affine, ``x * (1 + scale) + shift``
  with bf16 shift/scale from ``scale_shift_table + embedded_timestep``, then
  ``proj_out``.

The AdaLN MLPs get fp32 inputs, so the reference's bf16 weights are promoted
and the MLPs run in fp32 (torch fp32 GEMMs, a few rows each).  ``patchify_proj``
and ``proj_out`` are plain bf16 linears (cuBLAS through torch); the LayerNorm +
modulate of the head is ``ltxq_adaln_modulate``.  RoPE tables are taken
precomputed (``Modality.positional_embeddings``, as the reference accepts
them) or built from ``Modality.positions`` (``ltxq.rope``, the reference's
``_prepare_positional_embeddings`` / ``_prepare_cross_positional_embeddings``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from . import kernels as K
from . import rope as R
from .block import AUDIO_22B, VIDEO_22B, BasicAVTransformerBlock, RowShard, StreamConfig, TransformerArgs

TIMESTEP_CHANNELS = 256  # PixArtAlphaCombinedTimestepSizeEmbeddings.time_proj (timestep_embedding.py:139)
LATENT_CHANNELS = 128    # model.py:521-523 (video and audio VAE latent channels)


def timestep_embedding(t: torch.Tensor, dim: int = TIMESTEP_CHANNELS, max_period: int = 10000) -> torch.Tensor:
    """Sinusoidal embedding of fp32 timesteps (N,) -> (N, dim) fp32, ordered
    [cos | sin] (get_timestep_embedding with flip_sin_to_cos=True and no
    frequency shift, timestep_embedding.py:8-58)."""
    half = dim // 2
    # the Python scalar enters the fp32 kernel as fp32 (no host->device copy,
    # so the call is CUDA-graph capturable)
    expo = torch.arange(half, dtype=torch.float32, device=t.device) * (-math.log(max_period))
    freq = torch.exp(expo / half)
    arg = t.float()[:, None] * freq[None, :]
    return torch.cat([torch.cos(arg), torch.sin(arg)], dim=-1)


@dataclass
class AdaLNSingle:
    """AdaLayerNormSingle (timestep_embedding.py:165-201): timestep embedding
    -> linear_1 -> SiLU -> linear_2 (the embedded timestep) -> SiLU -> linear
    (``n`` rows of ``dim``).  Weights are kept in fp32."""

    w1: torch.Tensor
    b1: torch.Tensor
    w2: torch.Tensor
    b2: torch.Tensor
    w: torch.Tensor
    b: torch.Tensor
    n: int

    PARAMS = ("emb.timestep_embedder.linear_1", "emb.timestep_embedder.linear_2", "linear")

    @classmethod
    def from_state(cls, state: dict, prefix: str, n: int) -> "AdaLNSingle":
        t = []
        for p in cls.PARAMS:
            t += [state[f"{prefix}.{p}.weight"].float().contiguous(), state[f"{prefix}.{p}.bias"].float().contiguous()]
        return cls(*t, n=n)

    def __call__(self, t: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """fp32 timesteps (N,) -> (emb (N, n * dim), embedded_timestep (N, dim))."""
        h = F.silu(F.linear(timestep_embedding(t), self.w1, self.b1))
        emb_t = F.linear(h, self.w2, self.b2)
        return F.linear(F.silu(emb_t), self.w, self.b), emb_t


@dataclass
class Modality:
    """One stream's model input (the reference's ``Modality``): bf16 latent
    (B, T, 128); fp32 timesteps (B,) or per token (B, T); text context (B, L,
    C_ctx); RoPE (cos, sin) tables for self-attention and for the
    cross-modal attention, or None to build them from ``positions`` (fp32
    token bounds (B, n_dims, T, 2), ``ltxq.rope.video_positions`` /
    ``audio_positions``); fp32 sigma (B,) (the timesteps when None)."""

    latent: torch.Tensor
    timesteps: torch.Tensor
    context: torch.Tensor
    positional_embeddings: tuple | None = None
    cross_positional_embeddings: tuple | None = None
    sigma: torch.Tensor | None = None
    context_mask: torch.Tensor | None = None
    enabled: bool = True
    positions: torch.Tensor | None = None


@dataclass
class _Stream:
    """The modules of one stream that live outside the blocks."""

    cfg: StreamConfig
    patchify_w: torch.Tensor
    patchify_b: torch.Tensor
    adaln: AdaLNSingle
    prompt_adaln: AdaLNSingle
    cross_ss_adaln: AdaLNSingle
    cross_gate_adaln: AdaLNSingle
    scale_shift_table: torch.Tensor
    proj_out_w: torch.Tensor
    proj_out_b: torch.Tensor


# cache / checkpoint prefixes of the non-block modules (model.py:640-712)
_PREFIXES = {
    "video": dict(patchify="patchify_proj", adaln="adaln_single", prompt="prompt_adaln_single",
                  cross_ss="av_ca_video_scale_shift_adaln_single", cross_gate="av_ca_a2v_gate_adaln_single",
                  table="scale_shift_table", proj_out="proj_out"),
    "audio": dict(patchify="audio_patchify_proj", adaln="audio_adaln_single", prompt="audio_prompt_adaln_single",
                  cross_ss="av_ca_audio_scale_shift_adaln_single", cross_gate="av_ca_v2a_gate_adaln_single",
                  table="audio_scale_shift_table", proj_out="audio_proj_out"),
}


def model_param_specs(video: StreamConfig = VIDEO_22B, audio: StreamConfig = AUDIO_22B,
                      in_channels: int = LATENT_CHANNELS, out_channels: int = LATENT_CHANNELS) -> dict:
    """Every non-block parameter: key -> shape (the reference's names)."""
    specs: dict[str, tuple[int, ...]] = {}
    for which, cfg in (("video", video), ("audio", audio)):
        p = _PREFIXES[which]
        d = cfg.dim
        specs[f"{p['patchify']}.weight"] = (d, in_channels)
        specs[f"{p['patchify']}.bias"] = (d,)
        for key, n in (("adaln", 9), ("prompt", 2), ("cross_ss", 4), ("cross_gate", 1)):
            pre = p[key]
            specs[f"{pre}.emb.timestep_embedder.linear_1.weight"] = (d, TIMESTEP_CHANNELS)
            specs[f"{pre}.emb.timestep_embedder.linear_1.bias"] = (d,)
            specs[f"{pre}.emb.timestep_embedder.linear_2.weight"] = (d, d)
            specs[f"{pre}.emb.timestep_embedder.linear_2.bias"] = (d,)
            specs[f"{pre}.linear.weight"] = (n * d, d)
            specs[f"{pre}.linear.bias"] = (n * d,)
        specs[p["table"]] = (2, d)
        specs[f"{p['proj_out']}.weight"] = (out_channels, d)
        specs[f"{p['proj_out']}.bias"] = (out_channels,)
    return specs


def _stream_from_state(state: dict, which: str, cfg: StreamConfig) -> _Stream:
    p = _PREFIXES[which]
    return _Stream(cfg=cfg,
                   patchify_w=state[f"{p['patchify']}.weight"].to(torch.bfloat16).contiguous(),
                   patchify_b=state[f"{p['patchify']}.bias"].to(torch.bfloat16).contiguous(),
                   adaln=AdaLNSingle.from_state(state, p["adaln"], 9),
                   prompt_adaln=AdaLNSingle.from_state(state, p["prompt"], 2),
                   cross_ss_adaln=AdaLNSingle.from_state(state, p["cross_ss"], 4),
                   cross_gate_adaln=AdaLNSingle.from_state(state, p["cross_gate"], 1),
                   scale_shift_table=state[p["table"]].float().contiguous(),
                   proj_out_w=state[f"{p['proj_out']}.weight"].to(torch.bfloat16).contiguous(),
                   proj_out_b=state[f"{p['proj_out']}.bias"].to(torch.bfloat16).contiguous())


@dataclass
class LTXAVModel:
    """LTXModel (AudioVideo): ``model(video, audio)`` -> (video velocity,
    audio velocity), bf16 (B, T, 128) and (B, A, 128).

    ``timestep_scale_multiplier`` (1000) and ``av_ca_timestep_scale_multiplier``
    (1000, the loader's default when the checkpoint config has none,
    generate.py:1675-1678) follow the reference's constructor."""

    blocks: list
    video: _Stream
    audio: _Stream
    timestep_scale_multiplier: float = 1000.0
    av_ca_timestep_scale_multiplier: float = 1000.0
    norm_eps: float = 1e-6
    use_double_precision_rope: bool = False  # the checkpoint config's frequencies_precision == "float64"
    shard: RowShard | None = field(default=None, repr=False)

    # ------------------------------------------------------------- building
    @classmethod
    def from_state(cls, blocks: list, state: dict, video: StreamConfig = VIDEO_22B, audio: StreamConfig = AUDIO_22B,
                   **kw) -> "LTXAVModel":
        return cls(blocks, _stream_from_state(state, "video", video), _stream_from_state(state, "audio", audio), **kw)

    @classmethod
    def from_cache(cls, cache_file, device="cuda", video: StreamConfig = VIDEO_22B,
                   audio: StreamConfig = AUDIO_22B, **kw) -> "LTXAVModel":
        """The model from the reference's transformer cache (single file or
        shards, ``metadata.json`` beside it)."""
        from pathlib import Path

        from . import cache as C

        cache_file = Path(cache_file)
        weights = C.load_cache_weights(cache_file, device)
        blocks = C.blocks_from_weights(weights, C.read_metadata(cache_file.parent), video, audio)
        return cls.from_state(blocks, weights, video, audio, **kw)

    @classmethod
    def random(cls, gen: torch.Generator, device, n_blocks: int = 48, mode: str = "mxfp8", bits: int = 8,
               video: StreamConfig = VIDEO_22B, audio: StreamConfig = AUDIO_22B, w_std: float = 0.02,
               **kw) -> "LTXAVModel":
        """Random-init model (blocks as ``BasicAVTransformerBlock.random``;
        non-block weights ~N(0, w_std), biases ~N(0, 0.01), output tables
        ~N(0, 0.1))."""
        blocks = [BasicAVTransformerBlock.random(gen, device, mode=mode, bits=bits, video=video, audio=audio)
                  for _ in range(n_blocks)]
        return cls.from_state(blocks, random_model_state(gen, device, video, audio, w_std), video, audio, **kw)

    # ------------------------------------------------------------- RoPE
    def rope_tables(self, which: str, positions: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Self-attention RoPE tables of the "video" or "audio" stream from
        its token bounds (``_prepare_positional_embeddings``, model.py:256-283:
        middle of each bound, max_pos (20, 2048, 2048) / (20,))."""
        cfg = self.video.cfg if which == "video" else self.audio.cfg
        max_pos = R.VIDEO_MAX_POS if which == "video" else R.AUDIO_MAX_POS
        return R.precompute_freqs_cis(positions, cfg.dim, R.THETA, max_pos, True, cfg.heads,
                                      self.use_double_precision_rope)

    def cross_rope_tables(self, positions: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Audio<->video cross-attention RoPE tables of a stream from the
        temporal bounds of its tokens (``_prepare_cross_positional_embeddings``,
        model.py:392-417): audio width and heads, max_pos (20,)."""
        a = self.audio.cfg
        return R.precompute_freqs_cis(positions[:, 0:1], a.dim, R.THETA, R.AUDIO_MAX_POS, True, a.heads,
                                      self.use_double_precision_rope)

    def positional_tables(self, video_positions: torch.Tensor, audio_positions: torch.Tensor):
        """(video, audio, video cross, audio cross) tables of a stage, for
        callers that precompute them once (``denoise_av``)."""
        return (self.rope_tables("video", video_positions), self.rope_tables("audio", audio_positions),
                self.cross_rope_tables(video_positions), self.cross_rope_tables(audio_positions))

    # ------------------------------------------------------------- forward
    def _prepare(self, s: _Stream, m: Modality, cross: Modality) -> TransformerArgs:
        """MultiModalTransformerArgsPreprocessor.prepare (model.py:445-505)."""
        if m.context_mask is not None:  # the reference's pipelines pass None (pipelines/common.py:242-249, 285-292)
            raise ValueError("text-context attention masks are not supported")
        if not m.enabled:
            raise ValueError("both streams run in every call: a disabled modality is not supported")
        b = m.latent.shape[0]
        pe, cpe = m.positional_embeddings, m.cross_positional_embeddings
        if pe is None or cpe is None:
            if m.positions is None:
                raise ValueError("Modality needs RoPE tables or positions")
            which = "video" if s is self.video else "audio"
            pe = pe if pe is not None else self.rope_tables(which, m.positions)
            cpe = cpe if cpe is not None else self.cross_rope_tables(m.positions)
        d = s.cfg.dim
        x = F.linear(m.latent.to(torch.bfloat16), s.patchify_w, s.patchify_b)
        ts = m.timesteps.float()
        scaled = (ts * self.timestep_scale_multiplier).reshape(-1)
        emb, emb_t = s.adaln(scaled)
        sigma = (m.sigma if m.sigma is not None else m.timesteps).float()
        sigma = sigma[:, 0] if sigma.dim() > 1 else sigma
        prompt, _ = s.prompt_adaln(sigma * self.timestep_scale_multiplier)
        css, _ = s.cross_ss_adaln(scaled)
        csig = (cross.sigma if cross.sigma is not None else cross.timesteps).float()
        csig = csig[:, 0] if csig.dim() > 1 else csig
        cgate, _ = s.cross_gate_adaln(csig * self.av_ca_timestep_scale_multiplier)
        return TransformerArgs(x=x, context=m.context.to(torch.bfloat16), timesteps=emb.view(b, -1, 9, d),
                               positional_embeddings=pe, embedded_timestep=emb_t.view(b, -1, d),
                               cross_positional_embeddings=cpe,
                               cross_scale_shift_timestep=css.view(b, -1, 4, d),
                               cross_gate_timestep=cgate.view(b, -1, 1, d),
                               prompt_timestep=prompt.view(b, -1, 2, d))

    def _output(self, s: _Stream, x: torch.Tensor, embedded: torch.Tensor) -> torch.Tensor:
        """_process_video_output / _process_audio_output (model.py:1312-1340)."""
        ss = (s.scale_shift_table[None, None] + embedded[:, :, None, :]).to(torch.bfloat16)
        y = K.adaln_modulate(x, ss[:, :, 1], ss[:, :, 0], self.norm_eps, norm="layer")
        return F.linear(y, s.proj_out_w, s.proj_out_b)

    def __call__(self, video: Modality, audio: Modality, shard: RowShard | None = None, perturbations=None):
        """(video velocity, audio velocity).  With a row shard, ``video``
        holds this rank's latent rows (and their RoPE rows); the video
        velocity keeps that split, the audio velocity is replicated.
        ``perturbations`` (``ltxq.perturbations.BatchedPerturbationConfig``)
        makes this the perturbed pass of STG guidance."""
        shard = shard if shard is not None else self.shard
        va = self._prepare(self.video, video, audio)
        aa = self._prepare(self.audio, audio, video)
        for i, blk in enumerate(self.blocks):
            skip = perturbations.skipped(i) if perturbations is not None else frozenset()
            va, aa = blk(va, aa, shard, skip)
        return self._output(self.video, va.x, va.embedded_timestep), self._output(self.audio, aa.x,
                                                                                  aa.embedded_timestep)


def random_model_state(gen: torch.Generator, device, video: StreamConfig = VIDEO_22B,
                       audio: StreamConfig = AUDIO_22B, w_std: float = 0.02) -> dict[str, torch.Tensor]:
    """Random non-block parameters in the reference's key scheme: weights
    bf16 ~N(0, w_std), biases bf16 ~N(0, 0.01), output tables fp32
    ~N(0, 0.1)."""
    out = {}
    for key, shape in model_param_specs(video, audio).items():
        t = torch.randn(*shape, generator=gen, device=device)
        if key.endswith("scale_shift_table"):
            out[key] = t * 0.1
        elif key.endswith(".bias"):
            out[key] = (t * 0.01).to(torch.bfloat16)
        else:
            out[key] = (t * w_std).to(torch.bfloat16)
    return out


class X0Model:
    """X0Model (model.py:1489-1540): the denoised predictions
    ``latent - timesteps * velocity`` (fp32, as the reference's bf16 latent
    and fp32 timesteps promote) instead of the velocities.  The denoise loop
    (``ltxq.denoise.denoise_av``) fuses this step into ``ltxq_denoise_update``;
    this wrapper serves callers that want the reference's interface."""

    def __init__(self, velocity_model):
        self.velocity_model = velocity_model

    @staticmethod
    def denoise(m: Modality, velocity: torch.Tensor) -> torch.Tensor:
        t = m.timesteps.float()
        t = t[:, None, None] if t.dim() == 1 else t[:, :, None]
        return m.latent - t * velocity

    def __call__(self, video: Modality, audio: Modality, shard: RowShard | None = None, perturbations=None):
        vv, av = self.velocity_model(video, audio, shard, perturbations)
        return self.denoise(video, vv), self.denoise(audio, av)
