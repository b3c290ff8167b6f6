"""The LTX-2 audio-video transformer block on the ltxq hot path.

``BasicAVTransformerBlock`` mirrors LTX_2_MLX/model/transformer/transformer.py
:160-674 (same sub-layer order, AdaLN table slicing and residual forms) with
every linear layer a quantized GEMM from the C ABI:

* the AdaLN modulate of a sub-layer's input is computed once
  (``ltxq_adaln_modulate``) and feeds one GEMM whose weight is the
  concatenation of the projections reading that input (self-attention
  Q|K|V|gate-logits; cross-attention Q|gate-logits on the query side and
  K|V on the context side).  Concatenating packed rows along the output
  dimension is exact: every row keeps its own groups;
* the residual updates are GEMM epilogues of ``to_out`` / ``project_out``:
  gated residual (transformer.py:40-50, 469, 610-627, 650) or the text
  cross-attention gate-then-add (transformer.py:387, 484);
* the FF sub-layer is one ``ltxq_feed_forward`` call (GELU in project_in's
  epilogue).

QK RMSNorm and split RoPE (attention.py:320-329, rope.py:53-90) are one
fused CUDA pass (``ltxq_qk_norm_rope``) reading the strided Q/K columns of
the fused projection output; scaled-dot-product attention
(attention.py:170-302) runs through torch (cuDNN flash SDPA).

Parameter names follow the reference's cache key scheme
(loader/transformer_cache.py:35-59): ``attn1.to_q``, ``audio_ff.project_out``, ...
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from . import kernels as K
from .quantized_linear import QuantizedLinear


@dataclass(frozen=True)
class StreamConfig:
    """TransformerConfig (transformer.py:113-122) of one stream."""

    dim: int
    heads: int
    d_head: int
    context_dim: int


VIDEO_22B = StreamConfig(4096, 32, 128, 4096)   # model.py:514-515, 622-627
AUDIO_22B = StreamConfig(2048, 32, 64, 2048)

ATTN_PROJECTIONS = ("to_q", "to_k", "to_v", "to_out", "to_gate_logits")


def attention_dims(name: str, v: StreamConfig, a: StreamConfig):
    """(query_dim, context_dim, heads, d_head) of each attention module
    (transformer.py:183-269)."""
    return {
        "attn1": (v.dim, v.dim, v.heads, v.d_head),
        "attn2": (v.dim, v.context_dim, v.heads, v.d_head),
        "audio_attn1": (a.dim, a.dim, a.heads, a.d_head),
        "audio_attn2": (a.dim, a.context_dim, a.heads, a.d_head),
        "audio_to_video_attn": (v.dim, a.dim, a.heads, a.d_head),
        "video_to_audio_attn": (a.dim, v.dim, a.heads, a.d_head),
    }[name]


def linear_specs(v: StreamConfig = VIDEO_22B, a: StreamConfig = AUDIO_22B) -> dict[str, tuple[int, int]]:
    """Every quantized linear of a block: base name -> (out, in), in the
    cache's ``_CACHE_QUANTIZED_BLOCK_LINEAR_BASES`` order."""
    specs: dict[str, tuple[int, int]] = {}
    for name in ("attn1", "attn2", "audio_attn1", "audio_attn2", "audio_to_video_attn", "video_to_audio_attn"):
        qd, cd, h, d = attention_dims(name, v, a)
        inner = h * d
        specs[f"{name}.to_q"] = (inner, qd)
        specs[f"{name}.to_k"] = (inner, cd)
        specs[f"{name}.to_v"] = (inner, cd)
        specs[f"{name}.to_out"] = (qd, inner)
        specs[f"{name}.to_gate_logits"] = (h, qd)
    specs["ff.project_in.proj"] = (4 * v.dim, v.dim)
    specs["ff.project_out"] = (v.dim, 4 * v.dim)
    specs["audio_ff.project_in.proj"] = (4 * a.dim, a.dim)
    specs["audio_ff.project_out"] = (a.dim, 4 * a.dim)
    return specs


def table_specs(v: StreamConfig = VIDEO_22B, a: StreamConfig = AUDIO_22B) -> dict[str, tuple[int, ...]]:
    """fp32 AdaLN tables and QK-norm weights (transformer.py:210-269)."""
    t = {
        "scale_shift_table": (9, v.dim),
        "audio_scale_shift_table": (9, a.dim),
        "prompt_scale_shift_table": (2, v.dim),
        "audio_prompt_scale_shift_table": (2, a.dim),
        "scale_shift_table_a2v_ca_audio": (5, a.dim),
        "scale_shift_table_a2v_ca_video": (5, v.dim),
    }
    for name in ("attn1", "attn2", "audio_attn1", "audio_attn2", "audio_to_video_attn", "video_to_audio_attn"):
        _, _, h, d = attention_dims(name, v, a)
        t[f"{name}.q_norm.weight"] = (h * d,)
        t[f"{name}.k_norm.weight"] = (h * d,)
    return t


@dataclass
class TransformerArgs:
    """Per-stream inputs (transformer.py:125-157); batch entries share the
    rows dimension (x is (B, T, C)).  AdaLN tensors are fp32 with a broadcast
    token dimension: timesteps (B, 1, 9, C), prompt_timestep (B, 1, 2, C),
    cross_scale_shift_timestep (B, 1, 4, C), cross_gate_timestep (B, 1, 1, C).
    RoPE tables are (cos, sin), each (B, H, T, D/2) fp32."""

    x: torch.Tensor
    context: torch.Tensor
    timesteps: torch.Tensor
    positional_embeddings: tuple | None = None
    context_mask: torch.Tensor | None = None
    embedded_timestep: torch.Tensor | None = None
    cross_positional_embeddings: tuple | None = None
    cross_scale_shift_timestep: torch.Tensor | None = None
    cross_gate_timestep: torch.Tensor | None = None
    enabled: bool = True
    prompt_timestep: torch.Tensor | None = None

    def replace(self, **kw) -> "TransformerArgs":
        d = dict(self.__dict__)
        d.update(kw)
        return TransformerArgs(**d)


def rms_norm_weighted(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """QK RMSNorm (attention.py:320-329): fp32 math, cast back to bf16."""
    xf = x.float()
    inv = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (xf * inv * w.float()).to(torch.bfloat16)


def apply_split_rope(x: torch.Tensor, pe: tuple, heads: int) -> torch.Tensor:
    """rope.py:53-90 on (B, T, H*D) with cos/sin (B, H, T, D/2) fp32 ->
    (B, T, H*D) bf16 (token-major, so that rows can be all-gathered)."""
    b, t, width = x.shape
    d = width // heads
    xh = x.view(b, t, heads, d).float()
    x1, x2 = xh[..., : d // 2], xh[..., d // 2:]
    cos, sin = (c.transpose(1, 2) for c in pe)
    out = torch.cat([x1 * cos - x2 * sin, x1 * sin + x2 * cos], dim=-1).to(torch.bfloat16)
    return out.reshape(b, t, width)


def _heads(x: torch.Tensor, heads: int) -> torch.Tensor:
    b, t, width = x.shape
    return x.view(b, t, heads, width // heads).transpose(1, 2)


@dataclass
class RowShard:
    """Video-token row sharding over a process group (one rank per GPU):
    every linear, modulate and residual is row-local; by default the
    attention K/V computed from video rows are all-gathered (NCCL over
    NVLink) before the attention that reads all video keys -- video
    self-attention and video->audio cross-attention (``self_attention`` and
    ``v2a`` select the other exchanges).  Audio and text rows are
    replicated."""

    group: object = None
    world: int = 1
    rank: int = 0
    overlap: bool = True  # run the all-gathers on a side stream (start_gather / finish_gather)
    # video self-attention exchange: "gather" (all-gather K/V, attend the
    # local query rows) or "head_parallel" (all-to-all Q/K/V, attend H/world
    # heads over all rows, all-to-all the output back)
    self_attention: str = "gather"
    # video->audio keys: "gather" (all-gather the video K/V) or "split_keys"
    # (attend the local rows, merge the partial outputs by log-sum-exp)
    v2a: str = "gather"
    # optional callable(kind, phase): called with phase 0 just before and 1
    # just after each point where the caller's stream waits for an exchange
    # ("wait": the join of a side-stream collective) or runs one in line
    # ("sync"); a timer records device events there (bench.py: exposed
    # exchange time per step)
    wait_probe: object = field(default=None, repr=False, compare=False)
    _comm: object = field(default=None, repr=False, compare=False)

    def _probe(self, kind: str, phase: int) -> None:
        if self.wait_probe is not None:
            self.wait_probe(kind, phase)

    def gather_rows(self, x: torch.Tensor) -> torch.Tensor:
        """(B, T_local, C) on every rank -> (B, world * T_local, C)."""
        if self.world == 1:
            return x
        return self.finish_gather(self.start_gather(x, overlap=False))[0]

    def start_gather(self, *xs: torch.Tensor, overlap: bool | None = None) -> "PendingGather":
        """Start the all-gathers of ``xs``.  With overlap, they run on a side
        stream forked from the current one, and the caller's stream goes on
        with independent work until ``finish_gather``.  Outputs are allocated
        on the caller's stream and the inputs stay referenced until then, so
        neither is recycled while the side stream uses them."""
        xs = tuple(x.contiguous() for x in xs)
        if self.world == 1:
            return PendingGather(xs, xs, None)
        import torch.distributed as dist

        outs = tuple(torch.empty((self.world * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
                     for x in xs)  # rank-major blocks
        use_side = self.overlap if overlap is None else overlap
        if not use_side:
            self._probe("sync", 0)
            for o, x in zip(outs, xs):
                dist.all_gather_into_tensor(o, x, group=self.group)
            self._probe("sync", 1)
            return PendingGather(outs, xs, None)
        if self._comm is None:
            self._comm = torch.cuda.Stream(device=xs[0].device)
        cur = torch.cuda.current_stream(xs[0].device)
        self._comm.wait_stream(cur)
        with torch.cuda.stream(self._comm):
            for o, x in zip(outs, xs):
                dist.all_gather_into_tensor(o, x, group=self.group)
        return PendingGather(outs, xs, self._comm)

    def all_to_all(self, x: torch.Tensor) -> torch.Tensor:
        """Equal-split all-to-all along dim 0 (block g goes to rank g)."""
        import torch.distributed as dist

        out = torch.empty_like(x)
        self._probe("sync", 0)
        dist.all_to_all_single(out, x, group=self.group)
        self._probe("sync", 1)
        return out

    def start_all_to_all(self, x: torch.Tensor) -> "PendingGather":
        """``all_to_all`` on the side stream; ``finish_all_to_all`` joins it."""
        import torch.distributed as dist

        x = x.contiguous()
        out = torch.empty_like(x)
        if not self.overlap:
            self._probe("sync", 0)
            dist.all_to_all_single(out, x, group=self.group)
            self._probe("sync", 1)
            return PendingGather((out,), None, None)
        if self._comm is None:
            self._comm = torch.cuda.Stream(device=x.device)
        self._comm.wait_stream(torch.cuda.current_stream(x.device))
        with torch.cuda.stream(self._comm):
            dist.all_to_all_single(out, x, group=self.group)
        return PendingGather((out,), (x,), self._comm)

    def finish_all_to_all(self, pending: "PendingGather") -> torch.Tensor:
        if pending.stream is not None:
            self._probe("wait", 0)
            torch.cuda.current_stream(pending.outs[0].device).wait_stream(pending.stream)
            self._probe("wait", 1)
        return pending.outs[0]

    def finish_gather(self, pending: "PendingGather") -> tuple:
        """Join the side stream and return the gathered (B, world * T, C)."""
        if self.world == 1:
            return pending.outs
        if pending.stream is not None:
            self._probe("wait", 0)
            torch.cuda.current_stream(pending.outs[0].device).wait_stream(pending.stream)
            self._probe("wait", 1)
        res = []
        for o, x in zip(pending.outs, pending.inputs):
            b, t = x.shape[0], x.shape[1]
            rest = tuple(x.shape[2:])
            if b == 1:
                res.append(o.view((1, self.world * t) + rest))
            else:
                res.append(o.view((self.world, b, t) + rest).transpose(0, 1).reshape((b, self.world * t) + rest))
        return tuple(res)


@dataclass
class PendingGather:
    """All-gathers in flight (``RowShard.start_gather``)."""

    outs: tuple
    inputs: tuple
    stream: object


def heads_to_ranks(x: torch.Tensor, world: int, heads: int) -> torch.Tensor:
    """(B, T_local, H*D) -> the all-to-all send layout [world, B, T_local,
    H/world, D]: block g holds the heads rank g attends over."""
    b, t, w = x.shape
    d = w // heads
    return x.view(b, t, world, heads // world, d).permute(2, 0, 1, 3, 4).contiguous()


def ranks_to_sequence(y: torch.Tensor) -> torch.Tensor:
    """All-to-all receive layout [world (source = token block), B, T_local,
    H/world, D] -> (B, H/world, world*T_local, D), tokens in global order."""
    w, b, t, h, d = y.shape
    return y.permute(1, 3, 0, 2, 4).reshape(b, h, w * t, d)


def sequence_to_ranks(o: torch.Tensor, world: int) -> torch.Tensor:
    """(B, H/world, T, D) attention output -> the send layout [world (dest =
    token block), B, H/world, T/world, D]."""
    b, h, t, d = o.shape
    return o.view(b, h, world, t // world, d).permute(2, 0, 1, 3, 4).contiguous()


def ranks_to_heads(y: torch.Tensor) -> torch.Tensor:
    """Receive layout [world (source = head group), B, H/world, T_local, D] ->
    (B, T_local, H*D) with head group g at heads g*H/world ..."""
    w, b, h, t, d = y.shape
    return y.permute(1, 3, 0, 2, 4).reshape(b, t, w * h * d)


def merge_attention_partials(outs: torch.Tensor, lses: torch.Tensor) -> torch.Tensor:
    """Softmax attention over a key set split into parts: outs [P, ..., Lq, D]
    (each part's normalized output) and lses [P, ..., Lq] (each part's
    natural-log sum of exp scores) -> the output over all keys,
    sum_p exp(lse_p - L) out_p with L = logsumexp_p(lse_p), in fp32."""
    lse = torch.logsumexp(lses, dim=0)
    w = torch.exp(lses - lse.unsqueeze(0)).unsqueeze(-1)
    return (w * outs.float()).sum(dim=0)


@dataclass
class QAttention:
    """Attention (attention.py:360-603) with fused quantized projections."""

    name: str
    heads: int
    d_head: int
    self_attention: bool
    q_proj: QuantizedLinear        # self: Q|K|V|gate ; cross: Q|gate
    kv_proj: QuantizedLinear | None  # cross: K|V over the context
    to_out: QuantizedLinear
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    eps: float = 1e-6
    # "sdpa": torch's scaled_dot_product_attention (cuDNN / flash kernels);
    # "native": this library's sm_100a kernel (ltxq_attention)
    kernel: str = "sdpa"

    def project(self, x_mod: torch.Tensor, ctx_mod: torch.Tensor | None):
        inner = self.heads * self.d_head
        y = self.q_proj(x_mod)
        if self.self_attention:
            q, k, v, gl = y[..., :inner], y[..., inner:2 * inner], y[..., 2 * inner:3 * inner], y[..., 3 * inner:]
        else:
            kv = self.kv_proj(ctx_mod)
            q, gl = y[..., :inner], y[..., inner:]
            k, v = kv[..., :inner], kv[..., inner:]
        return q, k, v, gl

    def core(self, q, k, v, gl, pe=None, k_pe=None, gather_kv: RowShard | None = None) -> torch.Tensor:
        """QK norm, RoPE, SDPA, per-head gate -> (B, T, inner) bf16.  With
        ``gather_kv`` the (rotated) K and V rows of every rank are
        all-gathered first."""
        q, k = self.norm_rope(q, k, pe, k_pe)
        if gather_kv is not None and gather_kv.world > 1:
            k, v = gather_kv.finish_gather(gather_kv.start_gather(k, v, overlap=False))
        return self.attend(q, k, v, gl)

    def norm_rope(self, q, k, pe=None, k_pe=None):
        """QK RMSNorm + split RoPE (attention.py:580-587, rope.py:53-90); Q and
        K of the same rows and tables (self-attention) in one pass."""
        if k_pe is None and q.shape == k.shape and (self.heads * self.d_head // 16) % 32 == 0:
            return K.qk_norm_rope_pair(q, k, self.q_norm, self.k_norm, self.heads, self.eps, pe)
        q = K.qk_norm_rope(q, self.q_norm, self.heads, self.eps, pe)
        k = K.qk_norm_rope(k, self.k_norm, self.heads, self.eps, (pe if k_pe is None else k_pe) if pe is not None else None)
        return q, k

    def attend(self, q, k, v, gl) -> torch.Tensor:
        """SDPA and the per-head gate of rotated Q, K and V."""
        if self.kernel == "native":
            return self._gate(K.attention(q, k, v, self.heads, 1.0 / math.sqrt(self.d_head)), gl)
        qh, kh, vh = _heads(q, self.heads), _heads(k, self.heads), _heads(v, self.heads)
        o = F.scaled_dot_product_attention(qh, kh, vh, scale=1.0 / math.sqrt(self.d_head))
        b, h, t, d = o.shape
        o = o.transpose(1, 2).reshape(b, t, h * d)
        return self._gate(o, gl)

    def _gate(self, o: torch.Tensor, gl: torch.Tensor):
        """The per-head output gate, written in to_out's MX input form where
        to_out runs block-scaled."""
        width = o.shape[-1]
        terms = self.to_out.mx_terms(o.numel() // width) if width % 128 == 0 else 0
        return K.head_gate(o, gl, self.heads, mx_terms=terms)  # gl: a column slice, read in place

    def attend_head_parallel(self, qkv_recv: torch.Tensor, gl, shard: "RowShard") -> torch.Tensor:
        """Row-sharded self-attention in head-parallel form: ``qkv_recv`` is
        the all-to-all of [world, 3, B, T_local, H/world, D] (Q, K, V of
        ``heads_to_ranks``; this rank now holds H/world heads over all T
        tokens); SDPA runs on those heads and a second all-to-all returns
        every rank its token rows.  Each rank sends and receives (world-1)/world
        of its own Q, K, V and output rows, instead of receiving every other
        rank's K and V."""
        q, k, v = (ranks_to_sequence(qkv_recv[:, i]) for i in range(3))
        o = F.scaled_dot_product_attention(q, k, v, scale=1.0 / math.sqrt(self.d_head))
        back = shard.all_to_all(sequence_to_ranks(o, shard.world))
        return self._gate(ranks_to_heads(back), gl)

    def attend_split_keys(self, q, k_local, v_local, gl, shard: "RowShard") -> torch.Tensor:
        """Attention of replicated queries over keys / values sharded by rows:
        each rank attends over its own rows (memory-efficient SDPA, which also
        returns the log-sum-exp), the small per-rank outputs are
        all-gathered and merged (``merge_attention_partials``)."""
        import torch.distributed as dist

        qh, kh, vh = _heads(q, self.heads), _heads(k_local, self.heads), _heads(v_local, self.heads)
        o, lse = torch.ops.aten._scaled_dot_product_efficient_attention(
            qh, kh, vh, None, True, 0.0, False, scale=1.0 / math.sqrt(self.d_head))[:2]
        lq = qh.shape[2]
        part = torch.cat([o.float().flatten(), lse[..., :lq].float().flatten()])
        parts = torch.empty(shard.world * part.numel(), dtype=part.dtype, device=part.device)
        shard._probe("sync", 0)
        dist.all_gather_into_tensor(parts, part, group=shard.group)  # flat: valid for NCCL and gloo
        shard._probe("sync", 1)
        parts = parts.view(shard.world, -1)
        n_o = o.numel()
        outs = parts[:, :n_o].view((shard.world,) + tuple(o.shape))
        lses = parts[:, n_o:].view((shard.world,) + tuple(o.shape[:-1]))
        merged = merge_attention_partials(outs, lses).to(torch.bfloat16)
        b, h, t, d = merged.shape
        return self._gate(merged.transpose(1, 2).reshape(b, t, h * d), gl)


def _cat_linears(parts: list[QuantizedLinear]) -> QuantizedLinear:
    """Concatenate quantized linears along the output dimension.  Exact: in the
    standard layout each packed row keeps its own groups; in the pretransposed
    layout (groups along the output dimension) every part's width is a whole
    number of groups, so its columns keep theirs."""
    p0 = parts[0]
    for p in parts[1:]:
        assert p.in_features == p0.in_features and p.mode == p0.mode and p.bits == p0.bits
        assert p.group_size == p0.group_size and p.pretransposed == p0.pretransposed
    dim = 1 if p0.pretransposed else 0
    if p0.pretransposed:
        assert all(p.out_features % p.group_size == 0 for p in parts)
    bias = None
    if any(p.bias is not None for p in parts):
        bias = torch.cat([p.bias if p.bias is not None else torch.zeros(p.out_features, dtype=torch.bfloat16,
                                                                         device=p.weight.device) for p in parts])
    return QuantizedLinear(
        torch.cat([p.weight for p in parts], dim), torch.cat([p.scales for p in parts], dim),
        torch.cat([p.biases for p in parts], dim) if p0.biases is not None else None, bias,
        group_size=p0.group_size, bits=p0.bits, mode=p0.mode, pretransposed=p0.pretransposed,
        in_features=p0.in_features, out_features=sum(p.out_features for p in parts))


class BasicAVTransformerBlock:
    """transformer.py:160-674 over quantized weights."""

    def __init__(self, linears: dict[str, QuantizedLinear], tables: dict[str, torch.Tensor],
                 video: StreamConfig = VIDEO_22B, audio: StreamConfig = AUDIO_22B, norm_eps: float = 1e-6):
        self.video_cfg, self.audio_cfg, self.norm_eps = video, audio, norm_eps
        self.linears = linears
        self.tables = {k: v.float().contiguous() for k, v in tables.items()}
        self.attn = {}
        for name in ("attn1", "attn2", "audio_attn1", "audio_attn2", "audio_to_video_attn", "video_to_audio_attn"):
            _, _, h, d = attention_dims(name, video, audio)
            l = {p: linears[f"{name}.{p}"] for p in ATTN_PROJECTIONS}
            self_attn = name in ("attn1", "audio_attn1")
            if self_attn:
                q_proj, kv_proj = _cat_linears([l["to_q"], l["to_k"], l["to_v"], l["to_gate_logits"]]), None
            else:
                q_proj = _cat_linears([l["to_q"], l["to_gate_logits"]])
                kv_proj = _cat_linears([l["to_k"], l["to_v"]])
            self.attn[name] = QAttention(name, h, d, self_attn, q_proj, kv_proj, l["to_out"],
                                         self.tables[f"{name}.q_norm.weight"], self.tables[f"{name}.k_norm.weight"],
                                         norm_eps)
        self.ff = (linears["ff.project_in.proj"], linears["ff.project_out"])
        self.audio_ff = (linears["audio_ff.project_in.proj"], linears["audio_ff.project_out"])
        # the fused projections own the packed rows now; drop the per-projection
        # copies so that a block holds its weights once
        self.linears = {k: v for k, v in linears.items()
                        if not k.endswith((".to_q", ".to_k", ".to_v", ".to_gate_logits"))}
        self.probe = None  # optional callable(tag) recording events around the FF project_in GEMM
        self._expanded: dict = {}  # AdaLN table rows broadcast to a timestep tensor's shape (_table_like)

    # -------------------------------------------------------------- building
    @classmethod
    def random(cls, gen: torch.Generator, device, mode: str = "affine", bits: int = 8, group_size: int | None = None,
               video: StreamConfig = VIDEO_22B, audio: StreamConfig = AUDIO_22B, w_std: float = 0.02,
               b_std: float = 0.01, t_std: float = 0.1) -> "BasicAVTransformerBlock":
        """Random-init block: weights ~N(0, w_std) quantized on the GPU, biases
        ~N(0, b_std), AdaLN tables ~N(0, t_std), QK-norm weights 1 + N(0, t_std)."""
        lin, tabs = cls.random_parts(gen, device, mode, bits, group_size, video, audio, w_std, b_std, t_std)
        return cls(lin, tabs, video, audio)

    @staticmethod
    def random_parts(gen: torch.Generator, device, mode: str = "affine", bits: int = 8, group_size: int | None = None,
                     video: StreamConfig = VIDEO_22B, audio: StreamConfig = AUDIO_22B, w_std: float = 0.02,
                     b_std: float = 0.01, t_std: float = 0.1, pretransposed: bool = False):
        """The per-projection quantized linears (cache base name ->
        QuantizedLinear) and fp32 tables of a random block."""
        lin = {}
        for name, (n, k) in linear_specs(video, audio).items():
            w = (torch.randn(n, k, generator=gen, device=device) * w_std).to(torch.bfloat16)
            b = (torch.randn(n, generator=gen, device=device) * b_std).to(torch.bfloat16)
            lin[name] = QuantizedLinear.from_linear(w, b, group_size=group_size, bits=bits, mode=mode,
                                                    pretransposed=pretransposed)
            del w
        tabs = {}
        for name, shape in table_specs(video, audio).items():
            t = torch.randn(*shape, generator=gen, device=device) * t_std
            tabs[name] = (1.0 + t) if name.endswith("norm.weight") else t
        return lin, tabs

    def quantized_modules(self) -> list[QuantizedLinear]:
        mods = list(self.linears.values())
        for at in self.attn.values():
            mods.append(at.q_proj)
            if at.kv_proj is not None:
                mods.append(at.kv_proj)
        return mods

    def set_compute(self, compute: str) -> "BasicAVTransformerBlock":
        """How every quantized GEMM of the block computes (``QuantizedLinear.
        set_compute``): "dequant", or "mx2" / "mx1" for the native block-scaled
        fp8 MMAs on mxfp8 weights."""
        for ql in self.quantized_modules():
            ql.set_compute(compute)
        return self

    def set_attention(self, core: str) -> "BasicAVTransformerBlock":
        """The attention core of every attention sub-layer: "sdpa" (torch's
        scaled_dot_product_attention, the default) or "native" (this
        library's sm_100a kernel, ``ltxq_attention``).  The row-sharded
        head-parallel and split-key forms keep torch's kernels."""
        if core not in ("sdpa", "native"):
            raise ValueError(f"unknown attention core {core!r}")
        for at in self.attn.values():
            at.kernel = core
        return self

    def nbytes(self) -> int:
        """Bytes of packed weights, group parameters and biases held."""
        total = 0
        for ql in self.quantized_modules():
            for t in (ql.weight, ql.scales, ql.biases, ql.bias):
                if t is not None:
                    total += t.numel() * t.element_size()
        return total

    # -------------------------------------------------------------- forward
    def _ada(self, table: str, ts: torch.Tensor, start: int, end: int):
        """get_ada_values (transformer.py:286-309) -> list of (B, 1, C) fp32:
        slices of the table + timestep rows that ``_ada_prepare`` added."""
        key = (table, id(ts))
        vals = self._ada_rows.get(key)
        if vals is None:
            vals = self.tables[table][None, None] + ts[:, :, :self.tables[table].shape[0]]
            self._ada_rows[key] = vals
        return [vals[:, :, i] for i in range(start, end)]  # views: the kernels take strided vectors

    def _table_like(self, table: str, rows: slice, like: torch.Tensor) -> torch.Tensor:
        """``tables[table][rows]`` broadcast to ``like``'s shape as a dense
        tensor, kept while ``tables[table]`` is the same tensor object (the
        entry holds it) and unmodified (its in-place version counter)."""
        t = self.tables[table]
        key = (table, rows.start, rows.stop, tuple(like.shape))
        hit = self._expanded.get(key)
        if hit is not None and hit[0] is t and hit[1] == t._version:
            return hit[2]
        e = t[rows][None, None].expand(like.shape).contiguous()
        self._expanded[key] = (t, t._version, e)
        return e

    def _ada_prepare(self, video: TransformerArgs, audio: TransformerArgs) -> None:
        """Every AdaLN table + timestep sum of this block call
        (get_ada_values / get_av_ca_ada_values, transformer.py:286-342, and
        the text-CA prompt rows, :379) in one multi-tensor fp32 add: the same
        elementwise adds as one ``table + timestep`` per table, one launch
        instead of eight.  Results go to ``_ada_rows`` under (table, id of
        the timestep tensor); a sum that does not fit (missing tensor, other
        dtype, per-token rows) is left to the caller's own add."""
        want = []
        for args, base, prompt, cross in ((video, "scale_shift_table", "prompt_scale_shift_table",
                                           "scale_shift_table_a2v_ca_video"),
                                          (audio, "audio_scale_shift_table", "audio_prompt_scale_shift_table",
                                           "scale_shift_table_a2v_ca_audio")):
            n = self.tables[base].shape[0]
            want += [(base, slice(0, n), args.timesteps, args.timesteps[:, :, :n] if args.timesteps is not None
                      else None),
                     (prompt, slice(0, 2), args.prompt_timestep, args.prompt_timestep),
                     (cross, slice(0, 4), args.cross_scale_shift_timestep, args.cross_scale_shift_timestep),
                     ((cross, "gate"), slice(4, 5), args.cross_gate_timestep, args.cross_gate_timestep)]
        lhs, rhs, keys = [], [], []
        for table, rows, src, ts in want:
            name = table[0] if isinstance(table, tuple) else table
            # per-batch rows (B, 1, R, C) only: per-token timesteps keep the broadcast add
            if (ts is None or name not in self.tables or ts.dtype != torch.float32 or not ts.is_contiguous()
                    or ts.dim() != 4 or ts.shape[1] != 1 or ts.shape[-2] != rows.stop - rows.start):
                continue
            lhs.append(self._table_like(name, rows, ts))
            rhs.append(ts)
            keys.append((table, id(src)))
        for key, val in zip(keys, torch._foreach_add(lhs, rhs) if lhs else ()):
            self._ada_rows[key] = val

    def __call__(self, video: TransformerArgs, audio: TransformerArgs, shard: RowShard | None = None,
                 skip: frozenset = frozenset()):
        """One block.  With ``shard``, ``video`` holds this rank's rows (and
        the matching rows of its RoPE tables); the result keeps that split.
        ``skip`` names attention sub-layers to leave out (``PerturbationType``
        values of ``ltxq.perturbations``: a perturbed pass for STG,
        transformer.py:429-444, 455-457, 496-497, 574-575, 603-604)."""
        eps = self.norm_eps
        self._ada_rows = {}  # (table, timestep tensor) -> all rows, for this call only
        self._ada_prepare(video, audio)
        vx, ax = video.x.contiguous(), audio.x.contiguous()
        run_v = "skip_video_self_attn" not in skip
        run_a = "skip_audio_self_attn" not in skip
        run_a2v = "skip_a2v_cross_attn" not in skip
        run_v2a = "skip_v2a_cross_attn" not in skip

        sharded = shard is not None and shard.world > 1
        # video self-attention (transformer.py:447-471).  In a row-sharded
        # run its exchange -- the K/V all-gather, or with self_attention =
        # "head_parallel" (and heads divisible by the ranks) the Q/K/V
        # all-to-all -- overlaps the audio self- and text cross-attention,
        # which read no video rows (same results: the two streams are
        # independent until the audio<->video cross-attention)
        at = self.attn["attn1"]
        head_par = sharded and shard.self_attention == "head_parallel" and at.heads % shard.world == 0
        pend = None
        if run_v:
            sh, sc, g = self._ada("scale_shift_table", video.timesteps, 0, 3)
            q, k, v, gl = at.project(self._mod(vx, sc, sh, at.q_proj), None)
            q, k = at.norm_rope(q, k, video.positional_embeddings)
            if head_par:  # head-parallel attention: Q/K/V all-to-all, then SDPA on H/world heads
                qkv = torch.stack([heads_to_ranks(t_, shard.world, at.heads) for t_ in (q, k, v)], dim=1)
                pend = shard.start_all_to_all(qkv)
            elif sharded:
                pend = shard.start_gather(k, v)

        # audio self-attention + text cross-attention (transformer.py:488-527)
        if run_a:
            sh_a, sc_a, g_a = self._ada("audio_scale_shift_table", audio.timesteps, 0, 3)
            at_a = self.attn["audio_attn1"]
            qa, ka, va, gla = at_a.project(self._mod(ax, sc_a, sh_a, at_a.q_proj), None)
            o = at_a.core(qa, ka, va, gla, audio.positional_embeddings)
            ax = at_a.to_out(o, residual=ax, gate=g_a)
        ax = self._text_ca(ax, audio, "audio_attn2", "audio_scale_shift_table", "audio_prompt_scale_shift_table")

        if run_v:
            if head_par:
                o = at.attend_head_parallel(shard.finish_all_to_all(pend), gl, shard)
            else:
                if pend is not None:
                    k, v = shard.finish_gather(pend)
                o = at.attend(q, k, v, gl)
            vx = at.to_out(o, residual=vx, gate=g)

        # video text cross-attention (transformer.py:344-387, 473-486)
        vx = self._text_ca(vx, video, "attn2", "scale_shift_table", "prompt_scale_shift_table")

        # audio <-> video cross attention (transformer.py:529-627); both read
        # the norms of vx / ax taken before either residual update.  The
        # video->audio K/V (video rows) gather overlaps the audio->video
        # attention.
        a_sc_a2v, a_sh_a2v, a_sc_v2a, a_sh_v2a = self._ada_cross("scale_shift_table_a2v_ca_audio", audio)
        g_v2a = self._cross_gate("scale_shift_table_a2v_ca_audio", audio)
        v_sc_a2v, v_sh_a2v, v_sc_v2a, v_sh_v2a = self._ada_cross("scale_shift_table_a2v_ca_video", video)
        g_a2v = self._cross_gate("scale_shift_table_a2v_ca_video", video)
        at = self.attn["audio_to_video_attn"]
        if run_a2v:
            q, k, v, gl = at.project(self._mod(vx, v_sc_a2v, v_sh_a2v, at.q_proj),
                                     self._mod(ax, a_sc_a2v, a_sh_a2v, at.kv_proj))
        at2 = self.attn["video_to_audio_attn"]
        split_keys = sharded and shard.v2a == "split_keys"
        pend2 = None
        if run_v2a:
            q2, k2, v2, gl2 = at2.project(self._mod(ax, a_sc_v2a, a_sh_v2a, at2.q_proj),
                                          self._mod(vx, v_sc_v2a, v_sh_v2a, at2.kv_proj))
            q2, k2 = at2.norm_rope(q2, k2, audio.cross_positional_embeddings, video.cross_positional_embeddings)
            pend2 = shard.start_gather(k2, v2) if sharded and not split_keys else None
        if run_a2v:
            o = at.core(q, k, v, gl, video.cross_positional_embeddings, audio.cross_positional_embeddings)
            vx = at.to_out(o, residual=vx, gate=g_a2v)
        # video feed-forward (transformer.py:629-650).  It reads vx after the
        # audio->video update and nothing of the video->audio attention (which
        # only updates ax, from norms taken before either update), so it runs
        # here: in a row-sharded run the video->audio K/V all-gather, started
        # above, overlaps the block's largest GEMMs.  Same results as the
        # reference's order.
        vx = self._ff(vx, video, "scale_shift_table", self.ff)
        # video->audio: the audio queries are on every rank, the video keys
        # are split by rows.  "split_keys": each rank attends over its rows
        # and the partial results merge by their log-sum-exp (a ~1 MB exchange
        # instead of an all-gather of the video K/V)
        if run_v2a:
            if split_keys:
                o2 = at2.attend_split_keys(q2, k2, v2, gl2, shard)
            else:
                if pend2 is not None:
                    k2, v2 = shard.finish_gather(pend2)
                o2 = at2.attend(q2, k2, v2, gl2)
            ax = at2.to_out(o2, residual=ax, gate=g_v2a)

        # audio feed-forward (transformer.py:652-668)
        ax = self._ff(ax, audio, "audio_scale_shift_table", self.audio_ff)
        return video.replace(x=vx), audio.replace(x=ax)

    def _ada_cross(self, table: str, args: TransformerArgs):
        """get_av_ca_ada_values (transformer.py:311-342) scale/shift rows."""
        t = self._ada_rows.get((table, id(args.cross_scale_shift_timestep)))
        if t is None:
            t = self.tables[table][:4][None, None] + args.cross_scale_shift_timestep
        return [t[:, :, i] for i in range(4)]

    def _cross_gate(self, table: str, args: TransformerArgs):
        """The audio<->video gate row (transformer.py:311-342, row 4)."""
        t = self._ada_rows.get(((table, "gate"), id(args.cross_gate_timestep)))
        if t is None:
            return self.tables[table][4][None, None] + args.cross_gate_timestep[:, :, 0]
        return t[:, :, 0]

    def _text_ca(self, x, args: TransformerArgs, name: str, table: str, prompt_table: str):
        """Text cross-attention (transformer.py:344-387).  The text context is
        the same on every rank and its K/V projection runs replicated:
        splitting it across 8 ranks and all-gathering the rows measured
        slower (the gathers' latency exceeded the ~0.1 ms of GEMM saved)."""
        eps = self.norm_eps
        sh_q, sc_q, g = self._ada(table, args.timesteps, 6, 9)
        kv = self._ada_rows.get((prompt_table, id(args.prompt_timestep)))
        if kv is None:
            kv = self.tables[prompt_table][None, None] + args.prompt_timestep
        shift_kv, scale_kv = kv[:, :, 0], kv[:, :, 1]
        at = self.attn[name]
        q, k, v, gl = at.project(self._mod(x, sc_q, sh_q, at.q_proj),
                                 self._mod(args.context, scale_kv, shift_kv, at.kv_proj, "none"))
        o = at.core(q, k, v, gl)
        return at.to_out(o, residual=x, gate=g, gate_then_add=True)

    def _mod(self, x, scale, shift, consumer: QuantizedLinear, norm: str = "rms"):
        """AdaLN modulate (transformer.py:21-37, 379) of rows that feed
        ``consumer``: written directly in the block-scaled GEMM's MX input
        form where that GEMM runs block-scaled (the same bits as splitting
        the bf16 result), else as bf16."""
        C = x.shape[-1]
        terms = consumer.mx_terms(x.numel() // C) if K.mx_output_ok(C) and x.dtype == torch.bfloat16 else 0
        return K.adaln_modulate(x, scale, shift, self.norm_eps, norm, mx_terms=terms)

    def _ff(self, x, args: TransformerArgs, table: str, ff):
        sh, sc, g = self._ada(table, args.timesteps, 3, 6)
        probe = self.probe if ff is self.ff else None
        a = self._mod(x, sc, sh, ff[0])
        if probe is not None:
            probe("ff_in_start")
        # GELU(project_in) passes to project_out in its MX input form when
        # both run block-scaled
        h_terms = ff[1].mx_terms(a.M) if isinstance(a, K.MXActivation) and ff[1].in_features % 128 == 0 else 0
        h = ff[0](a, gelu=True, mx_out=h_terms)
        if probe is not None:
            probe("ff_in_end")
        return ff[1](h, residual=x, gate=g)
