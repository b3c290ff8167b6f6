"""The reference's quantized transformer cache, read and written on the
B200 side.

Format (LTX_2_MLX/loader/transformer_cache.py):

* files: ``<dir>/transformer.safetensors``, or shards beside it named
  ``transformer-00000.safetensors``, ``transformer-00001.safetensors``, ...
  (``_cache_shard_path`` :91-94); a writer starts a new shard once the
  current one holds >= 4 GiB (``_TRANSFORMER_SHARD_LIMIT_BYTES`` :85,
  :1217-1220); a reader merges every shard (``_load_cache_weights``
  :113-125);
* quantized block linears (``_CACHE_QUANTIZED_BLOCK_LINEAR_BASES`` :35-59)
  are stored as ``__quant__.transformer_blocks.{i}.{base}.weight`` (uint32
  packed codes), ``.scales`` (bf16 for affine, uint8 E8M0 for mxfp8) and,
  for affine only, ``.biases`` (:1255-1267); the linear's bias stays
  unquantized under its plain key ``transformer_blocks.{i}.{base}.bias``;
* every other parameter keeps its plain MLX key, e.g.
  ``transformer_blocks.{i}.scale_shift_table`` (fp32) or
  ``transformer_blocks.{i}.attn1.q_norm.weight``;
* in the ``mxfp8-blocks-pretranspose`` mode the quantized arrays are those
  of W^T (:1240-1244);
* ``metadata.json`` beside the cache holds the build payload
  (``_cache_payload`` :453-524): ``schema_version``, the source checkpoint's
  signature (resolved path, size, mtime in ns), ``include_audio``, the
  layout specs, ``transformer_cache_quantize`` and, when overridden,
  ``transformer_cache_quantize_group_size`` / ``_bits``, and
  ``fp8_dequant_policy`` for FP8 checkpoints.  A cache is valid when that
  file equals the payload expected for the current settings
  (``_metadata_matches`` :979-985); its directory is
  ``<root>/<checkpoint stem>-<first 20 hex digits of the payload's SHA-256>``
  (``transformer_cache_paths`` :711-758, ``_payload_digest`` :542-544).

safetensors itself is the public format (8-byte little-endian header length,
a JSON header mapping names to dtype / shape / byte range plus an optional
``__metadata__`` string map, then the raw little-endian data); it is read
and written here directly (``LTX_2_MLX/safetensors_header.py`` does the same
for headers), zero-copy through ``numpy.memmap``.
"""

from __future__ import annotations

import hashlib
import json
import os
import re
import struct
import warnings
from pathlib import Path

import numpy as np
import torch

QUANT_KEY_PREFIX = "__quant__."
SHARD_LIMIT_BYTES = 4 * 1024 ** 3
CACHE_SCHEMA_VERSION = 1
QUANTIZE_OFF, QUANTIZE_MXFP8_BLOCKS, QUANTIZE_MXFP8_BLOCKS_PRETRANSPOSE = (
    "off", "mxfp8-blocks", "mxfp8-blocks-pretranspose")
ATTENTION_MODULES = ("attn1", "attn2", "audio_attn1", "audio_attn2", "audio_to_video_attn", "video_to_audio_attn")
ATTENTION_PROJECTIONS = ("to_q", "to_k", "to_v", "to_out", "to_gate_logits")
QUANTIZED_BLOCK_LINEAR_BASES = tuple(f"{m}.{p}" for m in ATTENTION_MODULES for p in ATTENTION_PROJECTIONS) + (
    "ff.project_in.proj", "ff.project_out", "audio_ff.project_in.proj", "audio_ff.project_out")

# safetensors dtype name <-> (numpy storage dtype, torch dtype)
_DTYPES = {
    "BOOL": (np.bool_, torch.bool),
    "U8": (np.uint8, torch.uint8),
    "I8": (np.int8, torch.int8),
    "I16": (np.int16, torch.int16),
    "U16": (np.uint16, torch.uint16),
    "F16": (np.float16, torch.float16),
    "BF16": (np.uint16, torch.bfloat16),
    "I32": (np.int32, torch.int32),
    "U32": (np.uint32, torch.uint32),
    "F32": (np.float32, torch.float32),
    "F64": (np.float64, torch.float64),
    "I64": (np.int64, torch.int64),
    "U64": (np.uint64, torch.uint64),
    "F8_E4M3": (np.uint8, torch.float8_e4m3fn),
}
_TORCH_TO_NAME = {v[1]: k for k, v in _DTYPES.items()}


# ----------------------------------------------------------------------- safetensors


def read_safetensors_header(path) -> dict:
    """The JSON header (tensor entries and ``__metadata__`` if present)."""
    with open(path, "rb") as f:
        raw = f.read(8)
        if len(raw) != 8:
            raise ValueError(f"{path}: not a safetensors file (short header length)")
        (n,) = struct.unpack("<Q", raw)
        size = os.fstat(f.fileno()).st_size
        if n > size - 8:
            raise ValueError(f"{path}: header length {n} exceeds the file")
        return json.loads(f.read(n).decode("utf-8"))


def read_safetensors_metadata(path) -> dict:
    return dict(read_safetensors_header(path).get("__metadata__", {}) or {})


def read_safetensors_dtypes(path) -> dict:
    return {k: v["dtype"] for k, v in read_safetensors_header(path).items() if k != "__metadata__"}


def load_safetensors(path, device=None, keys=None) -> dict[str, torch.Tensor]:
    """Tensors of a safetensors file (all, or ``keys``), zero-copy views of a
    memory map when ``device`` is None, else copied to ``device``."""
    header = read_safetensors_header(path)
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
    base = 8 + n
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    out = {}
    for name, ent in header.items():
        if name == "__metadata__" or (keys is not None and name not in keys):
            continue
        if ent["dtype"] not in _DTYPES:
            raise ValueError(f"{path}: {name}: unsupported dtype {ent['dtype']}")
        np_dt, t_dt = _DTYPES[ent["dtype"]]
        b0, b1 = ent["data_offsets"]
        shape = tuple(ent["shape"])
        count = int(np.prod(shape)) if shape else 1
        if b1 - b0 != count * np.dtype(np_dt).itemsize:
            raise ValueError(f"{path}: {name}: byte range does not match shape {shape}")
        arr = np.frombuffer(mm, dtype=np_dt, count=count, offset=base + b0).reshape(shape)
        with warnings.catch_warnings():  # read-only memory map: torch warns about writes it will not see
            warnings.simplefilter("ignore", UserWarning)
            if t_dt is torch.bfloat16:
                t = torch.from_numpy(arr.view(np.int16)).view(torch.bfloat16)
            elif t_dt is torch.float8_e4m3fn:
                t = torch.from_numpy(arr).view(torch.float8_e4m3fn)
            else:
                t = torch.from_numpy(arr)
        out[name] = t.to(device) if device is not None else t
    return out


def save_safetensors(path, tensors: dict[str, torch.Tensor], metadata: dict[str, str] | None = None) -> None:
    """Write ``tensors`` (any device) as one safetensors file, atomically
    (a temporary file beside it, renamed into place)."""
    path = Path(path)
    header: dict = {}
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    blobs, off = [], 0
    for name in sorted(tensors):
        t = tensors[name].detach().contiguous().cpu()
        if t.dtype not in _TORCH_TO_NAME:
            raise ValueError(f"{name}: unsupported dtype {t.dtype}")
        raw = t.reshape(-1).view(torch.uint8).numpy().tobytes() if t.numel() else b""
        header[name] = {"dtype": _TORCH_TO_NAME[t.dtype], "shape": list(t.shape),
                        "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header, separators=(",", ":")).encode("utf-8")
    h += b" " * ((8 - len(h) % 8) % 8)
    tmp = path.parent / f".{path.stem}.tmp{path.suffix}"
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)
    os.replace(tmp, path)


# ----------------------------------------------------------------------- cache files


def cache_shard_path(cache_file, index: int) -> Path:
    cache_file = Path(cache_file)
    return cache_file.with_name(f"{cache_file.stem}-{index:05d}{cache_file.suffix}")


def existing_cache_shards(cache_file) -> list[Path]:
    cache_file = Path(cache_file)
    pat = re.compile(re.escape(cache_file.stem) + r"-[0-9]+" + re.escape(cache_file.suffix) + "$")
    return sorted(p for p in cache_file.parent.iterdir() if pat.match(p.name))


def load_cache_weights(cache_file, device=None) -> dict[str, torch.Tensor]:
    """The whole cache, single file or shards merged."""
    cache_file = Path(cache_file)
    if cache_file.exists():
        return load_safetensors(cache_file, device)
    shards = existing_cache_shards(cache_file)
    if not shards:
        raise FileNotFoundError(f"No cache at {cache_file} and no shards beside it.")
    merged: dict[str, torch.Tensor] = {}
    for s in shards:
        merged.update(load_safetensors(s, device))
    return merged


def write_cache_weights(cache_file, tensors: dict[str, torch.Tensor],
                        shard_limit_bytes: int = SHARD_LIMIT_BYTES) -> list[Path]:
    """Write ``tensors`` as shards beside ``cache_file`` (a new shard starts
    once the current one holds >= ``shard_limit_bytes``); removes an old
    single file or old shards first.  Returns the shard paths."""
    cache_file = Path(cache_file)
    cache_file.parent.mkdir(parents=True, exist_ok=True)
    if cache_file.exists():
        cache_file.unlink()
    for s in existing_cache_shards(cache_file):
        s.unlink()
    paths, cur, cur_bytes = [], {}, 0
    for name in tensors:
        if cur and cur_bytes >= shard_limit_bytes:
            paths.append(cache_shard_path(cache_file, len(paths)))
            save_safetensors(paths[-1], cur)
            cur, cur_bytes = {}, 0
        cur[name] = tensors[name]
        cur_bytes += tensors[name].numel() * tensors[name].element_size()
    if cur:
        paths.append(cache_shard_path(cache_file, len(paths)))
        save_safetensors(paths[-1], cur)
    return paths


def default_cache_root() -> Path:
    """default_transformer_cache_root (transformer_cache.py:359-372):
    $LTX_MLX_WEIGHTS_CACHE_DIR, else $LTX_MLX_TRANSFORMER_CACHE_DIR, else
    ~/.cache/ltx-2-mlx/weights-cache."""
    env = os.environ.get("LTX_MLX_WEIGHTS_CACHE_DIR") or os.environ.get("LTX_MLX_TRANSFORMER_CACHE_DIR")
    return Path(env).expanduser() if env else Path.home() / ".cache" / "ltx-2-mlx" / "weights-cache"


def file_signature(path) -> dict:
    """The source signature of a payload (transformer_cache.py:375-382)."""
    resolved = Path(path).expanduser().resolve()
    st = resolved.stat()
    return {"path": str(resolved), "size": st.st_size, "mtime_ns": st.st_mtime_ns}


def payload_digest(payload: dict) -> str:
    """First 20 hex digits of the SHA-256 of the compact, key-sorted JSON."""
    encoded = json.dumps(payload, sort_keys=True, separators=(",", ":")).encode("utf-8")
    return hashlib.sha256(encoded).hexdigest()[:20]


def safe_stem(path) -> str:
    stem = Path(path).stem
    safe = "".join(ch if ch.isalnum() or ch in ("-", "_", ".") else "_" for ch in stem)
    return safe[:80] or "transformer"


def transformer_cache_payload(weights_path, include_audio: bool = True,
                              transformer_cache_quantize: str = QUANTIZE_OFF, group_size: int | None = None,
                              bits: int | None = None) -> dict:
    """The payload the reference expects for a cache of ``weights_path``
    built with these settings and no layout or FF-quantization overrides
    (``_cache_payload``, transformer_cache.py:453-524)."""
    if transformer_cache_quantize not in (QUANTIZE_OFF, QUANTIZE_MXFP8_BLOCKS, QUANTIZE_MXFP8_BLOCKS_PRETRANSPOSE):
        raise ValueError(f"Unsupported transformer cache quantization mode: {transformer_cache_quantize}")
    payload = {"schema_version": CACHE_SCHEMA_VERSION, "source": file_signature(weights_path),
               "include_audio": include_audio, "video_ff_layout_specs": [], "video_ff_layout_layers": [],
               "video_attn_layout_specs": [], "video_attn_layout_layers": []}
    if transformer_cache_quantize != QUANTIZE_OFF:
        payload["transformer_cache_quantize"] = transformer_cache_quantize
        if group_size is not None:
            payload["transformer_cache_quantize_group_size"] = group_size
        if bits is not None:
            payload["transformer_cache_quantize_bits"] = bits
    try:
        if any(d in ("F8_E4M3", "F8_E5M2") for d in read_safetensors_dtypes(weights_path).values()):
            payload["fp8_dequant_policy"] = 2
    except Exception:  # an unreadable source fails later, in the build, with its own error
        pass
    return payload


def transformer_cache_paths(weights_path, cache_root=None, **settings) -> tuple[Path, Path, dict]:
    """(cache file, metadata file, expected payload) where the reference
    keeps the cache of ``weights_path`` for ``settings`` (the keyword
    arguments of ``transformer_cache_payload``)."""
    payload = transformer_cache_payload(weights_path, **settings)
    root = Path(cache_root).expanduser() if cache_root else default_cache_root()
    d = root / f"{safe_stem(weights_path)}-{payload_digest(payload)}"
    return d / "transformer.safetensors", d / "metadata.json", payload


def cache_is_valid(cache_file, expected_payload: dict) -> bool:
    """The cache exists (single file or shards) and its metadata equals the
    expected payload (``_cache_artifacts_exist`` / ``_metadata_matches``)."""
    cache_file = Path(cache_file)
    if not cache_file.parent.is_dir() or not (cache_file.exists() or existing_cache_shards(cache_file)):
        return False
    try:
        return json.loads((cache_file.parent / "metadata.json").read_text()) == expected_payload
    except (OSError, json.JSONDecodeError):
        return False


def cache_payload(transformer_cache_quantize: str = QUANTIZE_OFF, group_size: int | None = None,
                  bits: int | None = None, **extra) -> dict:
    """The quantization fields of the cache's metadata payload."""
    if transformer_cache_quantize not in (QUANTIZE_OFF, QUANTIZE_MXFP8_BLOCKS, QUANTIZE_MXFP8_BLOCKS_PRETRANSPOSE):
        raise ValueError(f"Unsupported transformer cache quantization mode: {transformer_cache_quantize}")
    payload = {"schema_version": CACHE_SCHEMA_VERSION, **extra}
    if transformer_cache_quantize != QUANTIZE_OFF:
        payload["transformer_cache_quantize"] = transformer_cache_quantize
        if group_size is not None:
            payload["transformer_cache_quantize_group_size"] = group_size
        if bits is not None:
            payload["transformer_cache_quantize_bits"] = bits
    return payload


def write_metadata(cache_dir, payload: dict) -> Path:
    p = Path(cache_dir) / "metadata.json"
    p.write_text(json.dumps(payload, indent=2, sort_keys=True))
    return p


def read_metadata(cache_dir) -> dict:
    p = Path(cache_dir) / "metadata.json"
    return json.loads(p.read_text()) if p.exists() else {}


# ----------------------------------------------------------------------- block state


def block_state(i: int, linears: dict, tables: dict) -> dict[str, torch.Tensor]:
    """Cache entries of block ``i`` from its per-projection quantized linears
    (base name -> ``QuantizedLinear``) and fp32 tables / norm weights."""
    out: dict[str, torch.Tensor] = {}
    for base in QUANTIZED_BLOCK_LINEAR_BASES:
        ql = linears[base]
        q = f"{QUANT_KEY_PREFIX}transformer_blocks.{i}.{base}"
        out[f"{q}.weight"] = ql.weight
        out[f"{q}.scales"] = ql.scales
        if ql.biases is not None:
            out[f"{q}.biases"] = ql.biases
        if ql.bias is not None:
            out[f"transformer_blocks.{i}.{base}.bias"] = ql.bias
    for name, t in tables.items():
        out[f"transformer_blocks.{i}.{name}"] = t
    return out


def split_block_state(weights: dict[str, torch.Tensor]) -> dict[int, dict]:
    """Group cache entries by block: {i: {"quant": {base: {weight, scales,
    biases?}}, "bias": {base: tensor}, "tables": {name: tensor}}}."""
    blocks: dict[int, dict] = {}
    for key, t in weights.items():
        quant = key.startswith(QUANT_KEY_PREFIX)
        k = key[len(QUANT_KEY_PREFIX):] if quant else key
        parts = k.split(".")
        if len(parts) < 3 or parts[0] != "transformer_blocks" or not parts[1].isdigit():
            continue
        i, rest = int(parts[1]), ".".join(parts[2:])
        b = blocks.setdefault(i, {"quant": {}, "bias": {}, "tables": {}})
        if quant:
            base, leaf = rest.rsplit(".", 1)
            b["quant"].setdefault(base, {})[leaf] = t
        elif rest.endswith(".bias") and rest[: -len(".bias")] in QUANTIZED_BLOCK_LINEAR_BASES:
            b["bias"][rest[: -len(".bias")]] = t
        else:
            b["tables"][rest] = t
    return blocks


def quantized_linears_from_state(state: dict, in_features: dict[str, int], payload: dict | None = None,
                                 mode: str | None = None, group_size: int | None = None,
                                 bits: int | None = None) -> dict:
    """``QuantizedLinear`` per base of one block's cache state.  The mode
    comes from the scales' dtype (uint8 E8M0 -> mxfp8, bf16 -> affine)
    unless given; group size and bits from the payload overrides or the
    reference's per-mode defaults (affine 64/4, mxfp8 32/8); ``in_features``
    maps base -> K (the packed arrays alone leave bits x K ambiguous)."""
    from .quantized_linear import QuantizedLinear, quant_defaults

    payload = payload or {}
    pretransposed = payload.get("transformer_cache_quantize") == QUANTIZE_MXFP8_BLOCKS_PRETRANSPOSE
    out = {}
    for base, arrs in state["quant"].items():
        m = mode or ("mxfp8" if arrs["scales"].dtype == torch.uint8 else "affine")
        k = in_features[base]
        rows, cols = arrs["weight"].shape
        if not pretransposed and bits is None and (cols * 32) % k == 0:
            bits_b = cols * 32 // k  # packed along K: the row length fixes the bit width
        else:
            bits_b = bits or payload.get("transformer_cache_quantize_bits") or payload.get("video_ff_quantize_bits")
        gs, b = quant_defaults(m, group_size or payload.get("transformer_cache_quantize_group_size")
                               or payload.get("video_ff_quantize_group_size")
                               or payload.get("block_linear_quantize_group_size"), bits_b)
        n = cols * 32 // b if pretransposed else rows
        out[base] = QuantizedLinear(arrs["weight"], arrs["scales"], arrs.get("biases"), state["bias"].get(base),
                                    group_size=gs, bits=b, mode=m, pretransposed=pretransposed,
                                    in_features=k, out_features=n)
    return out


def blocks_from_cache(cache_file, device="cuda", video=None, audio=None, blocks=None):
    """``BasicAVTransformerBlock`` list from a cache on disk (single file or
    shards, ``metadata.json`` beside it when present)."""
    cache_file = Path(cache_file)
    return blocks_from_weights(load_cache_weights(cache_file, device), read_metadata(cache_file.parent), video,
                               audio, blocks)


def blocks_from_weights(weights: dict[str, torch.Tensor], payload: dict | None = None, video=None, audio=None,
                        blocks=None):
    """``BasicAVTransformerBlock`` list from loaded cache entries (keys of
    other modules are ignored)."""
    from .block import AUDIO_22B, VIDEO_22B, BasicAVTransformerBlock, linear_specs

    video, audio = video or VIDEO_22B, audio or AUDIO_22B
    by_block = split_block_state(weights)
    kdims = {base: k for base, (_, k) in linear_specs(video, audio).items()}
    idx = sorted(by_block) if blocks is None else list(blocks)
    out = []
    for i in idx:
        st = by_block[i]
        missing = [b for b in QUANTIZED_BLOCK_LINEAR_BASES if b not in st["quant"]]
        if missing:
            raise ValueError(f"cache block {i}: missing quantized linears {missing[:4]}")
        lin = quantized_linears_from_state(st, kdims, payload)
        out.append(BasicAVTransformerBlock(lin, st["tables"], video, audio))
    return out
