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
