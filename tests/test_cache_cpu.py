"""CPU checks of the cache reader / writer (ltxq.cache) against the
reference's cache format: safetensors files (header, ``__metadata__``,
dtypes), sharding beside ``transformer.safetensors``, the
``__quant__.transformer_blocks.{i}.{base}`` key scheme and the metadata
payload fields (LTX_2_MLX/loader/transformer_cache.py; the reference's
tests/test_safetensors_header.py and tests/test_transformer_cache.py cover
the same behaviour on MLX)."""

import json
import struct
import types

import numpy as np
import pytest
import torch

from ltxq import cache as C


def test_metadata_and_dtypes_roundtrip(tmp_path):
    p = tmp_path / "t.safetensors"
    C.save_safetensors(p, {"w": torch.zeros(2, 3), "b": torch.ones(3, dtype=torch.bfloat16)},
                       metadata={"model_version": "2.3.0", "config": '{"x": 1}'})
    meta = C.read_safetensors_metadata(p)
    assert meta == {"model_version": "2.3.0", "config": '{"x": 1}'}
    assert C.read_safetensors_dtypes(p) == {"w": "F32", "b": "BF16"}
    header = C.read_safetensors_header(p)
    assert "w" in header and "b" in header


def test_metadata_empty_when_absent(tmp_path):
    p = tmp_path / "n.safetensors"
    C.save_safetensors(p, {"w": torch.zeros(1)})
    assert C.read_safetensors_metadata(p) == {}


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16, torch.uint8, torch.int32,
                                   torch.uint32, torch.int64, torch.float8_e4m3fn, torch.bool])
def test_tensor_roundtrip(tmp_path, dtype):
    g = torch.Generator().manual_seed(3)
    if dtype == torch.bool:
        t = torch.rand(5, 7, generator=g) > 0.5
    elif dtype in (torch.uint8, torch.int32, torch.uint32, torch.int64):
        t = torch.randint(0, 250, (5, 7), generator=g).to(dtype)
    else:
        t = torch.randn(5, 7, generator=g).to(dtype)
    p = tmp_path / "r.safetensors"
    C.save_safetensors(p, {"t": t, "scalar": torch.tensor(2.5), "empty": torch.zeros(0, 4)})
    back = C.load_safetensors(p)
    assert back["t"].dtype == dtype and back["t"].shape == t.shape
    assert torch.equal(back["t"].view(torch.uint8), t.view(torch.uint8))
    assert back["scalar"].shape == () and float(back["scalar"]) == 2.5
    assert back["empty"].shape == (0, 4)


def test_reads_a_file_it_did_not_write(tmp_path):
    """A file laid out by hand from the format description (unsorted keys,
    space padding, metadata first) reads back correctly."""
    a = np.arange(6, dtype=np.float32).reshape(2, 3)
    b = np.array([0x3F80, 0x4000], dtype=np.uint16)  # bf16 1.0, 2.0
    header = {"__metadata__": {"k": "v"},
              "zeta": {"dtype": "BF16", "shape": [2], "data_offsets": [24, 28]},
              "alpha": {"dtype": "F32", "shape": [2, 3], "data_offsets": [0, 24]}}
    h = json.dumps(header).encode() + b"   "
    p = tmp_path / "hand.safetensors"
    p.write_bytes(struct.pack("<Q", len(h)) + h + a.tobytes() + b.tobytes())
    t = C.load_safetensors(p)
    assert torch.equal(t["alpha"], torch.from_numpy(a))
    assert t["zeta"].dtype == torch.bfloat16 and t["zeta"].float().tolist() == [1.0, 2.0]
    assert C.read_safetensors_metadata(p) == {"k": "v"}


def test_sharded_cache_reload(tmp_path):
    cache_file = tmp_path / "transformer.safetensors"
    C.save_safetensors(C.cache_shard_path(cache_file, 0), {"transformer_blocks.0.weight": torch.tensor([1.0])})
    C.save_safetensors(C.cache_shard_path(cache_file, 1), {"transformer_blocks.1.weight": torch.tensor([2.0])})
    assert [p.name for p in C.existing_cache_shards(cache_file)] == ["transformer-00000.safetensors",
                                                                     "transformer-00001.safetensors"]
    w = C.load_cache_weights(cache_file)
    assert float(w["transformer_blocks.1.weight"]) == 2.0


def test_writer_shards_at_the_limit(tmp_path):
    cache_file = tmp_path / "transformer.safetensors"
    tensors = {f"transformer_blocks.{i}.w": torch.full((256,), float(i)) for i in range(10)}  # 1 KiB each
    paths = C.write_cache_weights(cache_file, tensors, shard_limit_bytes=3000)
    assert len(paths) == 4  # a new shard once one holds >= 3000 bytes: 3 + 3 + 3 + 1 tensors
    back = C.load_cache_weights(cache_file)
    assert set(back) == set(tensors)
    assert all(torch.equal(back[k], tensors[k]) for k in tensors)
    C.save_safetensors(cache_file, {"x": torch.zeros(1)})
    C.write_cache_weights(cache_file, {"y": torch.ones(1)})  # replaces the single file and old shards
    assert not cache_file.exists() and len(C.existing_cache_shards(cache_file)) == 1


def test_payload_keys_quant_group_overrides():
    a = C.cache_payload(C.QUANTIZE_MXFP8_BLOCKS, group_size=32)
    b = C.cache_payload(C.QUANTIZE_MXFP8_BLOCKS, group_size=64)
    assert a["transformer_cache_quantize_group_size"] == 32
    assert b["transformer_cache_quantize_group_size"] == 64
    assert a != b
    assert "transformer_cache_quantize" not in C.cache_payload(C.QUANTIZE_OFF)
    with pytest.raises(ValueError):
        C.cache_payload("mxfp4-everything")


def test_block_state_key_scheme_roundtrip():
    def ql(n, k, affine):
        return types.SimpleNamespace(weight=torch.zeros(n, k // 4, dtype=torch.int32),
                                     scales=torch.zeros(n, k // (64 if affine else 32),
                                                        dtype=torch.bfloat16 if affine else torch.uint8),
                                     biases=torch.zeros(n, k // 64, dtype=torch.bfloat16) if affine else None,
                                     bias=torch.zeros(n, dtype=torch.bfloat16))

    lin = {b: ql(64, 128, b.startswith("ff")) for b in C.QUANTIZED_BLOCK_LINEAR_BASES}
    tabs = {"scale_shift_table": torch.zeros(9, 64), "attn1.q_norm.weight": torch.ones(64)}
    st = C.block_state(3, lin, tabs)
    assert "__quant__.transformer_blocks.3.attn1.to_q.weight" in st
    assert "__quant__.transformer_blocks.3.ff.project_in.proj.biases" in st
    assert "__quant__.transformer_blocks.3.attn1.to_q.biases" not in st  # mxfp8: no biases
    assert "transformer_blocks.3.audio_ff.project_out.bias" in st
    assert "transformer_blocks.3.scale_shift_table" in st
    assert len([k for k in st if k.startswith("__quant__.")]) == 34 * 2 + 2  # + ff.project_in/out biases
    back = C.split_block_state(st)[3]
    assert set(back["quant"]) == set(C.QUANTIZED_BLOCK_LINEAR_BASES)
    assert set(back["bias"]) == set(C.QUANTIZED_BLOCK_LINEAR_BASES)
    assert set(back["tables"]) == set(tabs)
