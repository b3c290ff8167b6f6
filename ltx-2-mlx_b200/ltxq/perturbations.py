"""Attention perturbations for STG (spatio-temporal guidance): the
reference's LTX_2_MLX/components/perturbations.py interface.

A perturbed transformer pass skips chosen attention sub-layers in chosen
blocks.  A block skips a sub-layer only when every sample of the batch is
perturbed for it (``BatchedPerturbationConfig.all_in_batch``, as the
reference's block does at model/transformer/transformer.py:429-444); the
skipped sub-layer leaves its stream's residual unchanged.
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import Enum


class PerturbationType(Enum):
    SKIP_A2V_CROSS_ATTN = "skip_a2v_cross_attn"
    SKIP_V2A_CROSS_ATTN = "skip_v2a_cross_attn"
    SKIP_VIDEO_SELF_ATTN = "skip_video_self_attn"
    SKIP_AUDIO_SELF_ATTN = "skip_audio_self_attn"


@dataclass(frozen=True)
class Perturbation:
    """Skip ``type`` in ``blocks`` (None: every block)."""

    type: PerturbationType
    blocks: list[int] | None = None

    def is_perturbed(self, perturbation_type: PerturbationType, block: int) -> bool:
        return self.type == perturbation_type and (self.blocks is None or block in self.blocks)


@dataclass(frozen=True)
class PerturbationConfig:
    """The perturbations of one sample."""

    perturbations: list[Perturbation] | None = None

    def is_perturbed(self, perturbation_type: PerturbationType, block: int) -> bool:
        return bool(self.perturbations) and any(p.is_perturbed(perturbation_type, block)
                                                for p in self.perturbations)

    @staticmethod
    def empty() -> "PerturbationConfig":
        return PerturbationConfig(perturbations=[])


@dataclass(frozen=True)
class BatchedPerturbationConfig:
    """One ``PerturbationConfig`` per batch sample."""

    perturbations: list[PerturbationConfig]

    def all_in_batch(self, perturbation_type: PerturbationType, block: int) -> bool:
        return all(p.is_perturbed(perturbation_type, block) for p in self.perturbations)

    def skipped(self, block: int) -> frozenset[str]:
        """The sub-layers block ``block`` skips (``PerturbationType`` values)."""
        return frozenset(t.value for t in PerturbationType if self.all_in_batch(t, block))

    @staticmethod
    def empty(batch_size: int) -> "BatchedPerturbationConfig":
        return BatchedPerturbationConfig(perturbations=[PerturbationConfig.empty() for _ in range(batch_size)])


def create_stg_perturbation(skip_video_self_attn: bool = True, blocks: list[int] | None = None) -> PerturbationConfig:
    """The usual STG perturbation: skip the video self-attention."""
    ps = [Perturbation(PerturbationType.SKIP_VIDEO_SELF_ATTN, blocks)] if skip_video_self_attn else []
    return PerturbationConfig(perturbations=ps)


def create_batched_stg_config(batch_size: int, skip_video_self_attn: bool = True,
                              blocks: list[int] | None = None) -> BatchedPerturbationConfig:
    return BatchedPerturbationConfig([create_stg_perturbation(skip_video_self_attn, blocks)] * batch_size)
