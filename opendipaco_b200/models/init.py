"""Warm start every bank module from a pretrained dense Llama-style model.

Reference: ``src/opendipaco/init.py:25-73``. Each expert of a level copies the
same pretrained layers (at ``offset_of_key``), so experts start identical and
diverge only through training. The embedding, final norm and LM head go to
every embed/head module.
"""

from __future__ import annotations

import torch
from torch import nn

from ..topology import PathTopology


def load_pretrained(source: str | nn.Module) -> nn.Module:
    if isinstance(source, str):
        from transformers import AutoModelForCausalLM

        return AutoModelForCausalLM.from_pretrained(source)
    return source


def _llama_parts(model: nn.Module):
    base = getattr(model, "model", model)
    try:
        return base.embed_tokens, base.layers, base.norm, getattr(model, "lm_head", None)
    except AttributeError as exc:  # pragma: no cover
        raise ValueError("warm-start expects a Llama-style model exposing model.embed_tokens, "
                         "model.layers and model.norm") from exc


@torch.no_grad()
def warm_start_modules(bank: dict[str, nn.Module], topology: PathTopology,
                       source: str | nn.Module) -> None:
    model = load_pretrained(source).eval()
    embed, layers, norm, lm_head = _llama_parts(model)
    if len(layers) < topology.total_layers:
        raise ValueError(f"pretrained model has {len(layers)} layers but the path needs "
                         f"{topology.total_layers}")
    for key, mod in bank.items():
        role = topology.role_of_key(key)
        if role == "embed":
            mod.embed_tokens.load_state_dict(embed.state_dict())
        elif role == "head":
            mod.norm.load_state_dict(norm.state_dict())
            if lm_head is not None:
                mod.lm_head.load_state_dict(lm_head.state_dict())
        else:
            off = topology.offset_of_key(key)
            for i, layer in enumerate(mod.layers):
                # HF layers carry the same parameter names as ours.
                layer.load_state_dict(layers[off + i].state_dict(), strict=False)
