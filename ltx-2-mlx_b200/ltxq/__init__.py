"""ltxq -- B200-native (sm_100a) quantized DiT-block hot path of LTX-2-MLX.

Host-side mirror of the reference's interfaces for the path:
  * ``ltxq.kernels.adaln_norm_fused`` / ``gated_add_fused``
    (LTX_2_MLX/kernels/fused_ops.py:237, 398)
  * ``ltxq.quantized_linear.QuantizedLinear`` (MLX nn.QuantizedLinear and
    loader/transformer_cache.py:177-193 _PretransposedQuantizedLinear)
  * ``ltxq.feed_forward.FeedForward`` (model/transformer/feed_forward.py)
  * ``ltxq.block.BasicAVTransformerBlock`` / ``TransformerArgs``
    (model/transformer/transformer.py), ``ltxq.block.RowShard`` (video rows
    over several GPUs)
  * ``ltxq.model.LTXAVModel`` (model/transformer/model.py LTXModel) and
    ``ltxq.denoise`` / ``ltxq.perturbations`` (the AV denoise loop, sigma
    schedules, guiders, STG perturbations of components/ and pipelines/)
  * ``ltxq.cache`` / ``ltxq.cache_build`` (loader/transformer_cache.py)
The block linears, modulates, gates and the denoise update run in
``libltxq.so`` (hand-written CUDA for sm_100a) through its C ABI
(include/ltxq.h); there is no CPU fallback.
"""

from . import _lib
from .feed_forward import FeedForward
from .kernels import adaln_modulate, adaln_norm_fused, gated_add_fused, head_gate
from .quantized_linear import QuantizedLinear, quant_defaults

__all__ = [
    "FeedForward",
    "QuantizedLinear",
    "adaln_modulate",
    "adaln_norm_fused",
    "gated_add_fused",
    "head_gate",
    "quant_defaults",
]


def library_path() -> str:
    return _lib.LIB_PATH
