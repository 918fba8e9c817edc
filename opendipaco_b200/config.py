"""Configuration dataclasses.

Field names, order and defaults are part of the public API *and* of the checkpoint
format: the run fingerprint is a hash of ``repr(config) + "||" + repr(diloco)``
(reference ``src/opendipaco/train/loop.py:119-122``), so a checkpoint written by the
reference framework loads here only if these dataclasses print identically. They
therefore mirror ``src/opendipaco/config.py:19-205`` field for field.

B200-specific execution knobs (kernel path, CUDA graphs, comm backend) do not live
here; they are engine arguments (:class:`opendipaco_b200.train.ExecOptions`) so
that they never perturb the fingerprint.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from math import prod

from .topology import PathTopology, Segment, Sharing


@dataclass
class BackboneConfig:
    """Shape of the Llama-style transformer one path realises."""

    vocab_size: int = 32000
    hidden_size: int = 896
    num_attention_heads: int = 16
    num_key_value_heads: int | None = None
    intermediate_size: int = 2432
    max_position_embeddings: int = 2048
    rope_theta: float = 10000.0
    rms_norm_eps: float = 1e-5
    attn_implementation: str = "sdpa"
    layers_per_level: list[int] = field(default_factory=lambda: [6, 6])

    def kv_heads(self) -> int:
        return self.num_key_value_heads or self.num_attention_heads

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    @property
    def num_levels(self) -> int:
        return len(self.layers_per_level)

    @property
    def total_layers(self) -> int:
        return sum(self.layers_per_level)


@dataclass
class SegmentSpec:
    """Body segment for the advanced ``DiPaCoConfig.body`` API."""

    layers: int
    num_experts: int = 1
    sharing: str = "shared"


@dataclass
class DiPaCoConfig:
    """Full DiPaCo model description (simple ``level_sizes`` or advanced ``body``)."""

    backbone: BackboneConfig = field(default_factory=BackboneConfig)
    level_sizes: list[int] = field(default_factory=lambda: [4, 4])
    embedding: str = "shared"
    head: str = "shared"
    tie_word_embeddings: bool = False
    body: list[SegmentSpec] | None = None
    identical_expert_init: bool = True
    sequence_length: int = 1024
    eval_sequence_length: int | None = None

    def __post_init__(self) -> None:
        if self.body is None:
            if len(self.level_sizes) != self.backbone.num_levels:
                raise ValueError(
                    f"level_sizes has {len(self.level_sizes)} levels but backbone "
                    f"layers_per_level has {self.backbone.num_levels}"
                )
            if any(k < 1 for k in self.level_sizes):
                raise ValueError("each level must have at least one expert")
        if self.eval_sequence_length is not None and self.eval_sequence_length < 1:
            raise ValueError("eval_sequence_length must be >= 1")

    @property
    def eval_seq_len(self) -> int:
        return self.eval_sequence_length or self.sequence_length

    def segments(self) -> list[Segment]:
        segs = [Segment("embed", 0, 1, Sharing(self.embedding))]
        if self.body is None:
            segs += [
                Segment("body", n, k, Sharing.SHARED)
                for k, n in zip(self.level_sizes, self.backbone.layers_per_level)
            ]
        else:
            segs += [Segment("body", s.layers, s.num_experts, Sharing(s.sharing)) for s in self.body]
        segs.append(Segment("head", 0, 1, Sharing(self.head)))
        return segs

    def build_topology(self) -> PathTopology:
        return PathTopology(segments=self.segments())

    @property
    def num_paths(self) -> int:
        if self.body is None:
            return prod(self.level_sizes)
        return prod(s.num_experts for s in self.body if s.num_experts > 1) or 1


@dataclass
class DiLoCoConfig:
    """Inner (AdamW) / outer (SGD-Nesterov) optimisation hyper-parameters."""

    inner_steps: int = 150
    inner_lr: float = 4e-4
    inner_betas: tuple[float, float] = (0.9, 0.95)
    inner_weight_decay: float = 0.1
    inner_grad_clip: float | None = 1.0
    inner_autocast: bool = False
    activation_checkpoint: bool = False
    loss_chunks: int = 1
    optim_8bit: bool = False
    dedup_private: bool = False
    inner_lr_schedule: str = "cosine"
    inner_warmup_steps: int = 0
    inner_min_lr_ratio: float = 0.1
    outer_lr: float = 0.7
    outer_momentum: float = 0.9
    outer_nesterov: bool = True
    shard_size_weighting: bool = True
    normalize_outer_delta: bool = False
    rescale_by_sqrt_sharing: bool = True
