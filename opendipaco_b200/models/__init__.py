"""Model family: Llama-style DiPaCo paths (embed -> experts -> head)."""

from .init import load_pretrained, warm_start_modules
from .llama import (
    Attention, BlockModule, DecoderLayer, EmbeddingModule, HeadModule, LevelModule, MLP,
    RMSNorm, apply_rope, flops_per_token, param_count_per_layer, rope_cos_sin,
)
from .path import PathModel, build_module_bank, build_path_model

__all__ = [
    "Attention", "BlockModule", "DecoderLayer", "EmbeddingModule", "HeadModule", "LevelModule",
    "MLP", "RMSNorm", "apply_rope", "rope_cos_sin", "flops_per_token", "param_count_per_layer",
    "PathModel", "build_module_bank", "build_path_model", "warm_start_modules", "load_pretrained",
]
