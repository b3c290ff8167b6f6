"""The reference's audio-video transformer block, restated in numpy.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Follows LTX_2_MLX/model/transformer/transformer.py:389-674
(BasicAVTransformerBlock.__call__), attention.py:528-603 (Attention.__call__:
gate logits, V, Q, K projections; QK RMSNorm; split RoPE; SDPA; per-head gate;
to_out) and rope.py:53-90 (split rotary embedding, fp32 cos/sin, cast back to
bf16), with the rounding points of ref_ops.  Weights are given already
dequantized (bf16 values) so that the same function checks any quantization.

``p`` maps the reference's parameter names (the cache's key scheme,
loader/transformer_cache.py:35-59) to arrays:
``attn1.to_q.weight``, ``attn1.to_q.bias``, ``attn1.q_norm.weight``, ...,
``ff.project_in.proj.weight``, ``scale_shift_table`` ...
"""

from __future__ import annotations

import numpy as np

from . import _par
from . import ref_ops as ro
from .bf16 import rbf16

ATTN_MODULES = ("attn1", "attn2", "audio_attn1", "audio_attn2", "audio_to_video_attn", "video_to_audio_attn")


def rms_norm_weighted(x, w, eps=1e-6):
    """``RMSNorm`` module (attention.py:320-329): ``mx.fast.rms_norm(x, w, eps)``
    (fp32 math) cast back to bf16."""
    x = np.asarray(x, np.float32)
    ms = (x.astype(np.float64) ** 2).mean(-1, keepdims=True).astype(np.float32)
    inv = (1.0 / np.sqrt((ms + np.float32(eps)).astype(np.float64))).astype(np.float32)
    return rbf16(x * inv * np.asarray(w, np.float32))


def apply_split_rope(x, cos, sin, heads):
    """rope.py:53-90 on (T, H*D) bf16 with cos/sin (H, T, D/2) fp32."""
    t, width = x.shape
    d = width // heads
    xh = np.asarray(x, np.float32).reshape(t, heads, d).transpose(1, 0, 2)
    x1, x2 = xh[..., : d // 2], xh[..., d // 2 :]
    out = np.concatenate([x1 * cos - x2 * sin, x1 * sin + x2 * cos], axis=-1)
    return rbf16(out.astype(np.float32)).transpose(1, 0, 2).reshape(t, width)


def _softmax_rows(s):
    """Row softmax in fp32 (max-subtracted), in place on a fresh array."""
    s = s - s.max(-1, keepdims=True)
    np.exp(s, out=s)
    s /= s.sum(-1, keepdims=True)
    return s


def sdpa(q, k, v, heads, max_scores: int = 1 << 28):
    """mx.fast.scaled_dot_product_attention, no mask: fp32 softmax, bf16 out.
    Heads are independent, so they are processed in groups whose score
    matrices hold at most ``max_scores`` fp32 values (same result, bounded
    memory at long sequences)."""
    tq, width = q.shape
    tk = k.shape[0]
    d = width // heads
    qh = np.asarray(q, np.float32).reshape(tq, heads, d).transpose(1, 0, 2)
    kh = np.asarray(k, np.float32).reshape(tk, heads, d).transpose(1, 0, 2)
    vh = np.asarray(v, np.float32).reshape(tk, heads, d).transpose(1, 0, 2)
    o = np.empty((heads, tq, d), np.float32)
    step = max(1, min(heads, max_scores // max(1, tq * tk)))
    for h0 in range(0, heads, step):
        sl = slice(h0, h0 + step)
        s = (qh[sl] @ kh[sl].transpose(0, 2, 1)) * np.float32(1.0 / np.sqrt(d))
        s = _par.chunked(_softmax_rows, s.reshape(-1, tk)).reshape(s.shape)
        o[sl] = s @ vh[sl]
    return rbf16(o).transpose(1, 0, 2).reshape(tq, width)


def attention(p, name, x, context=None, pe=None, k_pe=None, heads=32, eps=1e-6):
    """Attention.__call__ (attention.py:528-603) for one batch row."""
    lin = lambda base, inp: ro.linear(inp, p[f"{name}.{base}.weight"], p.get(f"{name}.{base}.bias"))
    ctx = x if context is None else context
    gate_logits = lin("to_gate_logits", x)
    v = lin("to_v", ctx)
    q = lin("to_q", x)
    k = lin("to_k", ctx)
    q = rms_norm_weighted(q, p[f"{name}.q_norm.weight"], eps)
    k = rms_norm_weighted(k, p[f"{name}.k_norm.weight"], eps)
    if pe is not None:
        q = apply_split_rope(q, pe[0], pe[1], heads)
        kp = pe if k_pe is None else k_pe
        k = apply_split_rope(k, kp[0], kp[1], heads)
    out = sdpa(q, k, v, heads)
    out = ro.head_gate(out, gate_logits, heads)
    return lin("to_out", out)


def ada(table, ts, start, end):
    """get_ada_values (transformer.py:286-309): fp32 table rows + timestep
    rows; ``ts`` is (rows, C) for the row, or (T, rows, C) per token."""
    ts = np.asarray(ts, np.float32)
    return [np.asarray(table[i], np.float32) + ts[..., i, :] for i in range(start, end)]


def block(p, video, audio, heads_v=32, heads_a=32, eps=1e-6, skip=frozenset()):
    """BasicAVTransformerBlock.__call__ for one batch row.  ``skip`` holds
    the perturbed sub-layers ("skip_video_self_attn", "skip_audio_self_attn",
    "skip_a2v_cross_attn", "skip_v2a_cross_attn"; transformer.py:429-444),
    which leave their stream's residual unchanged.

    video / audio: dicts with x (T, C), context (L, Cctx), timesteps (9, C)
    or per token (T, 9, C), pe (cos, sin), cross_pe (cos, sin), cross_ss
    (4, C) or (T, 4, C), cross_gate (1, C), prompt (2, C).  Returns (vx, ax)."""
    vx, ax = video["x"], audio["x"]
    # video self-attention (transformer.py:447-471)
    if "skip_video_self_attn" not in skip:
        sh, sc, g = ada(p["scale_shift_table"], video["timesteps"], 0, 3)
        nv = ro.adaln(vx, sc, sh, eps)
        vx = ro.gated_add(vx, attention(p, "attn1", nv, pe=video["pe"], heads=heads_v, eps=eps), g)
    # video text cross-attention (transformer.py:344-387, 473-486)
    sh_q, sc_q, g = ada(p["scale_shift_table"], video["timesteps"], 6, 9)
    kv = ada(p["prompt_scale_shift_table"], video["prompt"], 0, 2)
    a_in = ro.adaln(vx, sc_q, sh_q, eps)
    enc = ro.modulate(video["context"], kv[1], kv[0])
    vx = ro.gate_then_add(vx, attention(p, "attn2", a_in, context=enc, heads=heads_v, eps=eps), g)
    # audio self-attention + text cross-attention (transformer.py:488-527)
    if "skip_audio_self_attn" not in skip:
        sh, sc, g = ada(p["audio_scale_shift_table"], audio["timesteps"], 0, 3)
        na = ro.adaln(ax, sc, sh, eps)
        ax = ro.gated_add(ax, attention(p, "audio_attn1", na, pe=audio["pe"], heads=heads_a, eps=eps), g)
    sh_q, sc_q, g = ada(p["audio_scale_shift_table"], audio["timesteps"], 6, 9)
    kv = ada(p["audio_prompt_scale_shift_table"], audio["prompt"], 0, 2)
    a_in = ro.adaln(ax, sc_q, sh_q, eps)
    enc = ro.modulate(audio["context"], kv[1], kv[0])
    ax = ro.gate_then_add(ax, attention(p, "audio_attn2", a_in, context=enc, heads=heads_a, eps=eps), g)
    # audio <-> video cross attention (transformer.py:529-627)
    vn3 = ro.rms_norm(vx, eps)
    an3 = ro.rms_norm(ax, eps)
    ta, tv = p["scale_shift_table_a2v_ca_audio"], p["scale_shift_table_a2v_ca_video"]
    a_sc_a2v, a_sh_a2v, a_sc_v2a, a_sh_v2a = ada(ta, audio["cross_ss"], 0, 4)
    g_v2a = ta[4] + np.asarray(audio["cross_gate"], np.float32)[..., 0, :]
    v_sc_a2v, v_sh_a2v, v_sc_v2a, v_sh_v2a = ada(tv, video["cross_ss"], 0, 4)
    g_a2v = tv[4] + np.asarray(video["cross_gate"], np.float32)[..., 0, :]
    vx_new = vx
    if "skip_a2v_cross_attn" not in skip:
        vxs = ro.modulate(vn3, v_sc_a2v, v_sh_a2v)
        axs = ro.modulate(an3, a_sc_a2v, a_sh_a2v)
        out = attention(p, "audio_to_video_attn", vxs, context=axs, pe=video["cross_pe"], k_pe=audio["cross_pe"],
                        heads=heads_a, eps=eps)
        vx_new = ro.gated_add(vx, out, g_a2v)
    if "skip_v2a_cross_attn" not in skip:
        axs = ro.modulate(an3, a_sc_v2a, a_sh_v2a)
        vxs = ro.modulate(vn3, v_sc_v2a, v_sh_v2a)
        out = attention(p, "video_to_audio_attn", axs, context=vxs, pe=audio["cross_pe"], k_pe=video["cross_pe"],
                        heads=heads_a, eps=eps)
        ax = ro.gated_add(ax, out, g_v2a)
    vx = vx_new
    # feed-forwards (transformer.py:629-668)
    sh, sc, g = ada(p["scale_shift_table"], video["timesteps"], 3, 6)
    vx = ro.ff_sublayer(vx, sc, sh, g, p["ff.project_in.proj.weight"], p["ff.project_in.proj.bias"],
                        p["ff.project_out.weight"], p["ff.project_out.bias"], eps)
    sh, sc, g = ada(p["audio_scale_shift_table"], audio["timesteps"], 3, 6)
    ax = ro.ff_sublayer(ax, sc, sh, g, p["audio_ff.project_in.proj.weight"], p["audio_ff.project_in.proj.bias"],
                        p["audio_ff.project_out.weight"], p["audio_ff.project_out.bias"], eps)
    return vx, ax
