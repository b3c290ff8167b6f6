"""CPU checks of the checkpoint side of the cache builder (ltxq.cache_build):
the reference's key mapping (loader/weight_converter.py:10-50) and its FP8
checkpoint handling (loader/transformer_cache.py:605-708), including the
reference test's known answer (tests/test_transformer_cache.py:64-95: E4M3
0x38 with weight_scale 2.0 loads as bf16 2.0)."""

import pytest
import torch

from ltxq import cache as C
from ltxq import cache_build as B


@pytest.mark.parametrize("src,want", [
    ("transformer_blocks.3.attn1.to_out.0.weight", "transformer_blocks.3.attn1.to_out.weight"),
    ("transformer_blocks.3.ff.net.0.proj.weight", "transformer_blocks.3.ff.project_in.proj.weight"),
    ("transformer_blocks.3.ff.net.2.bias", "transformer_blocks.3.ff.project_out.bias"),
    ("transformer_blocks.0.audio_ff.net.0.proj.weight", "transformer_blocks.0.audio_ff.project_in.proj.weight"),
    ("transformer_blocks.0.audio_ff.net.2.weight", "transformer_blocks.0.audio_ff.project_out.weight"),
    ("transformer_blocks.1.scale_shift_table", "transformer_blocks.1.scale_shift_table"),
    ("video_embeddings_connector.layer.weight", None),
])
def test_key_mapping(src, want):
    assert B.convert_checkpoint_key(src) == want


def test_audio_keys_skipped_without_audio():
    assert B.convert_checkpoint_key("transformer_blocks.0.audio_attn1.to_q.weight", include_audio=False) is None
    assert B.convert_checkpoint_key("transformer_blocks.0.audio_to_video_attn.to_q.weight", include_audio=False) is None
    assert B.convert_checkpoint_key("transformer_blocks.0.attn1.to_q.weight", include_audio=False) is not None


def test_fp8_checkpoint_dequant_and_companions(tmp_path):
    p = tmp_path / "ckpt.safetensors"
    code = torch.tensor([[0x38, 0xB8], [0x40, 0x00]], dtype=torch.uint8).view(torch.float8_e4m3fn)
    C.save_safetensors(p, {
        "layer.weight": code,
        "layer.weight_scale": torch.tensor(2.0),
        "layer.input_scale": torch.tensor(0.5),
        "layer.comfy_quant": torch.tensor([123], dtype=torch.uint8),
        "plain.weight": code,  # FP8 without a scale: exact decode
        "other.shift_scale": torch.tensor([1.0, 2.0]),  # a *_scale with no FP8 base stays
    })
    items = dict(B.iter_checkpoint_weights(p))
    assert set(items) == {"layer.weight", "plain.weight", "other.shift_scale"}
    assert items["layer.weight"].dtype == torch.bfloat16
    assert items["layer.weight"].float().tolist() == [[2.0, -2.0], [4.0, 0.0]]
    assert items["plain.weight"].float().tolist() == [[1.0, -1.0], [2.0, 0.0]]
    assert items["other.shift_scale"].tolist() == [1.0, 2.0]


def test_e5m2_rejected(tmp_path):
    p = tmp_path / "e5.safetensors"
    C.save_safetensors(p, {"w": torch.zeros(2, dtype=torch.uint8)})
    import json
    import struct

    raw = p.read_bytes()
    (n,) = struct.unpack("<Q", raw[:8])
    h = json.loads(raw[8:8 + n])
    h["w"]["dtype"] = "F8_E5M2"
    hb = json.dumps(h).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    p.write_bytes(struct.pack("<Q", len(hb)) + hb + raw[8 + n:])
    with pytest.raises(ValueError, match="E5M2"):
        list(B.iter_checkpoint_weights(p))


def _tiny_checkpoint(path, fp8=False):
    import torch

    from ltxq import cache as C

    t = {"model.diffusion_model.transformer_blocks.0.scale_shift_table": torch.zeros(9, 8),
         "model.diffusion_model.patchify_proj.weight": torch.ones(8, 4, dtype=torch.bfloat16)}
    if fp8:
        t["model.diffusion_model.proj_out.weight"] = torch.zeros(4, 8, dtype=torch.float8_e4m3fn)
    C.save_safetensors(path, t)
    return path


def test_transformer_cache_payload_matches_the_reference_fields(tmp_path):
    """_cache_payload (transformer_cache.py:453-524) for the default layouts:
    schema, source signature, include_audio, empty layout specs, the
    quantization fields only when set (tests/test_transformer_cache.py:98-115
    of the reference: group sizes change the payload and its digest), and
    the FP8 dequant policy for FP8 checkpoints."""
    import os

    from ltxq import cache as C

    ck = _tiny_checkpoint(tmp_path / "ckpt.safetensors")
    p = C.transformer_cache_payload(ck, include_audio=False)
    st = os.stat(ck)
    assert p == {"schema_version": 1, "source": {"path": str(ck.resolve()), "size": st.st_size,
                                                 "mtime_ns": st.st_mtime_ns},
                 "include_audio": False, "video_ff_layout_specs": [], "video_ff_layout_layers": [],
                 "video_attn_layout_specs": [], "video_attn_layout_layers": []}
    a = C.transformer_cache_payload(ck, transformer_cache_quantize="mxfp8-blocks", group_size=32)
    b = C.transformer_cache_payload(ck, transformer_cache_quantize="mxfp8-blocks", group_size=64)
    assert a["transformer_cache_quantize_group_size"] == 32 and b["transformer_cache_quantize_group_size"] == 64
    assert a != b and C.payload_digest(a) != C.payload_digest(b)
    assert "fp8_dequant_policy" not in a
    f8 = _tiny_checkpoint(tmp_path / "f8.safetensors", fp8=True)
    assert C.transformer_cache_payload(f8)["fp8_dequant_policy"] == 2
    with pytest.raises(ValueError):
        C.transformer_cache_payload(ck, transformer_cache_quantize="int4")


def test_cache_paths_and_digest(tmp_path, monkeypatch):
    import hashlib

    from ltxq import cache as C

    assert C.payload_digest({"b": [], "a": 1}) == hashlib.sha256(b'{"a":1,"b":[]}').hexdigest()[:20]
    assert C.safe_stem("/x/LTX 2.3 (22b).safetensors") == "LTX_2.3__22b_"
    ck = _tiny_checkpoint(tmp_path / "ckpt.safetensors")
    monkeypatch.setenv("LTX_MLX_WEIGHTS_CACHE_DIR", str(tmp_path / "root"))
    f, meta, payload = C.transformer_cache_paths(ck, transformer_cache_quantize="mxfp8-blocks")
    assert f.parent == tmp_path / "root" / f"ckpt-{C.payload_digest(payload)}"
    assert f.name == "transformer.safetensors" and meta == f.parent / "metadata.json"
    monkeypatch.delenv("LTX_MLX_WEIGHTS_CACHE_DIR")
    monkeypatch.setenv("LTX_MLX_TRANSFORMER_CACHE_DIR", str(tmp_path / "legacy"))
    assert C.default_cache_root() == tmp_path / "legacy"


def test_ensure_transformer_cache_builds_reuses_and_follows_the_source(tmp_path):
    """mode "off" needs no GPU: the first call builds (metadata = the
    expected payload), the second reuses, a changed checkpoint gets a new
    digest directory."""
    import os
    import time

    from ltxq import cache as C
    from ltxq import cache_build as CB

    ck = _tiny_checkpoint(tmp_path / "ckpt.safetensors")
    root = tmp_path / "root"
    f1 = CB.ensure_transformer_cache(ck, root, mode="off", device="cpu")
    _, _, payload = C.transformer_cache_paths(ck, root, transformer_cache_quantize="off")
    assert C.cache_is_valid(f1, payload)
    assert C.read_metadata(f1.parent) == payload
    w = C.load_cache_weights(f1)
    assert set(w) == {"transformer_blocks.0.scale_shift_table", "patchify_proj.weight"}
    shard = C.existing_cache_shards(f1)[0]
    mtime = shard.stat().st_mtime_ns
    assert CB.ensure_transformer_cache(ck, root, mode="off", device="cpu") == f1
    assert shard.stat().st_mtime_ns == mtime  # reused, not rebuilt
    time.sleep(0.01)
    os.utime(ck)  # a new source signature
    f2 = CB.ensure_transformer_cache(ck, root, mode="off", device="cpu")
    assert f2.parent != f1.parent and C.cache_is_valid(f2, C.transformer_cache_paths(ck, root)[2])
    assert not C.cache_is_valid(f1, C.transformer_cache_paths(ck, root)[2])
