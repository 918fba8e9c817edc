"""VRAM planning and measurement (reference ``src/opendipaco/train/memory.py``).

``vram_breakdown`` counts a path's parameters on the ``meta`` device (exact
parameter/optimizer terms, coarse activations); ``measure_peak`` measures one real
round on CUDA. ``fused_breakdown`` adds the B200 fused executor's actual resident
layout (fp32 master + fp32 grads + AdamW m/v + bf16 working copy per owned path,
plus the per-step activation arena), which is what sizes shards for 180 GB HBM.
"""

from __future__ import annotations

import torch

from ..models.path import build_module_bank, build_path_model
from ..topology import is_private_key

BLOCK_ACT_FACTOR = 16


def _count_params(config):
    with torch.device("meta"):
        bank = build_module_bank(config)
        pm = build_path_model(config, config.build_topology().path_from_index(0), bank,
                              deepcopy=False)

    def numel(params, seen):
        n = 0
        for p in params:
            if id(p) not in seen:
                seen.add(id(p))
                n += p.numel()
        return n

    total = numel(pm.parameters(), set())
    private, seen = 0, set()
    for k, mod in pm.modules_by_key().items():
        if is_private_key(k):
            private += numel(mod.parameters(), seen)
    return total, private, numel(pm.embed.parameters(), set()), numel(pm.head.parameters(), set())


def vram_breakdown(config, *, batch_size: int, seq_len: int, autocast: bool = False,
                   checkpoint: bool = False, master_bytes: int = 4,
                   chunked_logits: bool = False) -> dict:
    total, private, _, _ = _count_params(config)
    act_b = 2 if autocast else 4
    depth = sum(config.backbone.layers_per_level)
    tokens = batch_size * seq_len
    params = total * master_bytes
    block = depth * tokens * config.backbone.hidden_size * act_b * (1 if checkpoint else BLOCK_ACT_FACTOR)
    logits = 0 if chunked_logits else tokens * config.backbone.vocab_size * act_b
    out = {"n_params": total, "n_private": private, "params": params, "global": params,
           "adam": 2 * params, "grads": params, "activations": block + logits, "logits": logits}
    out["total"] = out["params"] + out["global"] + out["adam"] + out["grads"] + out["activations"]
    return out


def fused_breakdown(config, *, paths_per_gpu: int, batch_size: int, seq_len: int) -> dict:
    """Resident bytes of the fused executor for ``paths_per_gpu`` owned paths."""
    total, _, _, _ = _count_params(config)
    bb = config.backbone
    m = batch_size * seq_len
    per_path = total * (4 + 4 + 4 + 4 + 2)       # master, grad, m, v, bf16 copy
    layers = sum(config.backbone.layers_per_level)
    qkv = (bb.num_attention_heads + 2 * bb.kv_heads()) * bb.head_dim
    act_layer = m * (bb.hidden_size * (4 + 2 + 2) + qkv * 2 + bb.hidden_size * 2
                     + 3 * bb.intermediate_size * 2) + m * 16
    act = layers * act_layer + m * bb.vocab_size * 2 + m * bb.hidden_size * 8
    return {"per_path_state": per_path, "activations_per_path": act,
            "total": paths_per_gpu * (per_path + act)}


def fits(breakdown: dict, budget_bytes: int) -> bool:
    return breakdown["total"] <= budget_bytes


def measure_peak(config, diloco, *, device: str, batch_size: int, seq_len: int,
                 seed: int = 0) -> int | None:
    if not (str(device).startswith("cuda") and torch.cuda.is_available()):
        return None
    from ..parallel.backend import LocalBackend
    from ..schedule.scheduler import AsyncScheduler
    from .loop import DiPaCoEngine

    torch.cuda.empty_cache()
    torch.cuda.reset_peak_memory_stats()
    eng = DiPaCoEngine(config, diloco, LocalBackend(config.build_topology()), device=device,
                       seed=seed, materialize="serial")
    worker = AsyncScheduler(eng, num_workers=1)
    g = torch.Generator().manual_seed(seed)
    shard = torch.randint(0, config.backbone.vocab_size, (max(2 * batch_size, 4), seq_len), generator=g)
    worker._train_path(config.build_topology().path_from_index(0), shard, batch_size, 0)
    return int(torch.cuda.max_memory_allocated())
