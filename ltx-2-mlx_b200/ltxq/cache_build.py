"""Building the reference's quantized transformer cache from a checkpoint.

Restates the checkpoint side of LTX_2_MLX/loader:

* key mapping (``weight_converter.py:10-50``, ``convert_pytorch_key_to_mlx``):
  checkpoint keys under ``model.diffusion_model.`` lose that prefix;
  ``to_out.0`` -> ``to_out``, ``ff.net.0.proj`` -> ``ff.project_in.proj``,
  ``ff.net.2`` -> ``ff.project_out`` (and the ``audio_ff`` forms); the text
  embeddings connectors are not transformer weights and are skipped; without
  ``include_audio`` every audio / cross-modal key is skipped;
* FP8 checkpoints (``transformer_cache.py:605-708``): ``F8_E4M3`` tensors
  decode exactly; one with a ``<key>_scale`` companion (``weight_scale``) is
  dequantized in fp32 as ``e4m3 * weight_scale`` and rounded once to bf16;
  ``weight_scale``, ``input_scale`` and ComfyUI ``comfy_quant`` companions
  are dropped; ``F8_E5M2`` is rejected;
* quantized block linears (``transformer_cache.py:1238-1267``): every
  ``transformer_blocks.{i}.{base}.weight`` of the 34 block-linear bases is
  quantized (here on the GPU, ``ltxq_quantize``) and stored under
  ``__quant__.transformer_blocks.{i}.{base}.{weight,scales[,biases]}``; the
  ``mxfp8-blocks-pretranspose`` mode quantizes W^T.  Other tensors keep their
  key and dtype.  The cache is sharded at 4 GiB and ``metadata.json`` holds
  the payload the reference expects for the same checkpoint and settings
  (``_cache_payload`` :453-524), so the reference accepts the cache as
  valid; ``ensure_transformer_cache`` (:1749-1812) reuses a valid cache or
  builds one in the digest-named directory the reference uses.

Beyond the reference's modes (off, mxfp8-blocks, mxfp8-blocks-pretranspose),
``affine=(bits, group_size)`` quantizes the block linears with MLX affine
int8 / int4 (the layout of benchmark configs 1-3 and 5); the payload then
records ``block_linear_quantize = "affine"`` with its bits and group size.
"""

from __future__ import annotations

import re
from pathlib import Path

import torch

from . import cache as C

CHECKPOINT_PREFIX = "model.diffusion_model."
_FP8 = ("F8_E4M3",)


def convert_checkpoint_key(key: str, include_audio: bool = True) -> str | None:
    """Checkpoint key (prefix already removed) -> the MLX model key, or None
    for keys the transformer does not hold."""
    if not include_audio and ("av_ca" in key or "a2v" in key or "audio" in key.lower()):
        return None
    if "video_embeddings_connector" in key or "audio_embeddings_connector" in key:
        return None
    key = re.sub(r"\.to_out\.0\.", ".to_out.", key)
    key = re.sub(r"(^|\.)ff\.net\.0\.proj\.", r"\1ff.project_in.proj.", key)
    key = re.sub(r"(^|\.)ff\.net\.2\.", r"\1ff.project_out.", key)
    key = re.sub(r"(^|\.)audio_ff\.net\.0\.proj\.", r"\1audio_ff.project_in.proj.", key)
    key = re.sub(r"(^|\.)audio_ff\.net\.2\.", r"\1audio_ff.project_out.", key)
    return key


def fp8_companions(header_dtypes: dict[str, str]):
    """(fp8 keys, weight_scale keys, input_scale keys, comfy_quant keys)."""
    fp8 = {k for k, d in header_dtypes.items() if d in _FP8}
    wscale = {k for k in header_dtypes if k.endswith("_scale") and k[: -len("_scale")] in fp8}
    iscale = {k[: -len(".weight")] + ".input_scale" for k in fp8 if k.endswith(".weight")}
    iscale &= set(header_dtypes)
    comfy = {k for k in header_dtypes if k.endswith(".comfy_quant") and k[: -len(".comfy_quant")] + ".weight" in fp8}
    return fp8, wscale, iscale, comfy


def iter_checkpoint_weights(path, device=None, value_dtype=torch.bfloat16):
    """(key, tensor) of a safetensors checkpoint with FP8 weights decoded
    (scaled ones in fp32, rounded once to ``value_dtype``) and their
    companions dropped."""
    dtypes = C.read_safetensors_dtypes(path)
    if any(d == "F8_E5M2" for d in dtypes.values()):
        raise ValueError("F8_E5M2 checkpoints are not supported (E4M3 only)")
    fp8, wscale, iscale, comfy = fp8_companions(dtypes)
    raw = C.load_safetensors(path)
    for key, t in raw.items():
        if key in wscale or key in iscale or key in comfy:
            continue
        if key in fp8:
            sk = key + "_scale"
            if sk in wscale:
                v = (t.to(device).float() * raw[sk].to(device).float()).to(value_dtype)
            else:
                v = t.to(device).to(value_dtype)  # E4M3 values are exact in bf16
            yield key, v
        else:
            yield key, t.to(device) if device is not None else t


def _block_linear(mlx_key: str):
    parts = mlx_key.split(".")
    if len(parts) < 5 or parts[0] != "transformer_blocks" or not parts[1].isdigit() or parts[-1] != "weight":
        return None
    base = ".".join(parts[2:-1])
    return (int(parts[1]), base) if base in C.QUANTIZED_BLOCK_LINEAR_BASES else None


def build_transformer_cache(checkpoint, cache_file, mode: str = C.QUANTIZE_MXFP8_BLOCKS,
                            affine: tuple[int, int] | None = None, include_audio: bool = True,
                            device="cuda", shard_limit_bytes: int = C.SHARD_LIMIT_BYTES) -> dict:
    """Write the cache of ``checkpoint`` (a safetensors file with
    ``model.diffusion_model.`` keys) beside ``cache_file``; returns the
    metadata payload.  ``affine=(bits, group_size)`` quantizes the block
    linears affine instead of mxfp8 (no reference mode: the payload adds
    ``block_linear_quantize`` keys)."""
    from .quantized_linear import QuantizedLinear

    if affine is not None and mode != C.QUANTIZE_OFF:
        raise ValueError("affine block quantization goes with mode='off' (the reference's modes are mxfp8)")
    quant = affine is not None or mode != C.QUANTIZE_OFF
    pretransposed = mode == C.QUANTIZE_MXFP8_BLOCKS_PRETRANSPOSE
    entries: dict[str, torch.Tensor] = {}
    for key, value in iter_checkpoint_weights(checkpoint, device):
        if not key.startswith(CHECKPOINT_PREFIX):
            continue
        mlx_key = convert_checkpoint_key(key[len(CHECKPOINT_PREFIX):], include_audio)
        if mlx_key is None:
            continue
        bl = _block_linear(mlx_key) if quant else None
        if bl is None:
            entries[mlx_key] = value
            continue
        i, base = bl
        w = value.to(device=device, dtype=torch.bfloat16)
        if affine is not None:
            ql = QuantizedLinear.from_linear(w, None, group_size=affine[1], bits=affine[0], mode="affine")
        else:
            ql = QuantizedLinear.from_linear(w, None, mode="mxfp8", pretransposed=pretransposed)
        q = f"{C.QUANT_KEY_PREFIX}transformer_blocks.{i}.{base}"
        entries[f"{q}.weight"] = ql.weight
        entries[f"{q}.scales"] = ql.scales
        if ql.biases is not None:
            entries[f"{q}.biases"] = ql.biases
    payload = C.transformer_cache_payload(checkpoint, include_audio=include_audio,
                                          transformer_cache_quantize=C.QUANTIZE_OFF if affine else mode)
    if affine is not None:
        payload.update(block_linear_quantize="affine", block_linear_quantize_bits=affine[0],
                       block_linear_quantize_group_size=affine[1])
    C.write_cache_weights(cache_file, entries, shard_limit_bytes)
    C.write_metadata(Path(cache_file).parent, payload)
    return payload


def ensure_transformer_cache(checkpoint, cache_root=None, mode: str = C.QUANTIZE_MXFP8_BLOCKS,
                             include_audio: bool = True, rebuild: bool = False, device="cuda",
                             shard_limit_bytes: int = C.SHARD_LIMIT_BYTES) -> Path:
    """The cache file of ``checkpoint`` for these settings: reused when its
    metadata matches the expected payload (the reference's cache_mode
    "auto"), else (or with ``rebuild``) built where the reference looks for
    it.  Returns the cache file path (single file or shard base name)."""
    cache_file, _, payload = C.transformer_cache_paths(checkpoint, cache_root, include_audio=include_audio,
                                                       transformer_cache_quantize=mode)
    if not rebuild and C.cache_is_valid(cache_file, payload):
        return cache_file
    got = build_transformer_cache(checkpoint, cache_file, mode=mode, include_audio=include_audio, device=device,
                                  shard_limit_bytes=shard_limit_bytes)
    if got != payload:  # the checkpoint changed while the cache was being built
        raise RuntimeError(f"{checkpoint} changed during the cache build")
    return cache_file
