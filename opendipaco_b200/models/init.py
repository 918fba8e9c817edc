"""Warm start of the module bank from a pretrained dense Llama-style model.

Every module takes its tensors from the pretrained model by name: the embedding
modules its token embedding; the head modules its final norm and LM head; an expert
of a level the pretrained layers at that level's depth offset. All experts of a level
therefore start identical and diverge only through training (the reference's
``src/opendipaco/init.py`` does the same). The pretrained model is a Hugging Face
``AutoModelForCausalLM`` (loaded by name) or any module with Llama parameter names,
with or without the leading ``model.``.
"""

from __future__ import annotations

import re

import torch
from torch import nn

from ..topology import PathTopology

_LAYER = re.compile(r"^layers\.(\d+)\.(.+)$")


def load_pretrained(source: str | nn.Module) -> nn.Module:
    if isinstance(source, str):
        from transformers import AutoModelForCausalLM

        return AutoModelForCausalLM.from_pretrained(source)
    return source


def _pretrained_tensors(model: nn.Module) -> dict[str, torch.Tensor]:
    """The model's tensors under Llama names without the ``model.`` prefix."""
    out = {}
    for name, t in model.state_dict().items():
        out[name[len("model."):] if name.startswith("model.") else name] = t
    if "embed_tokens.weight" not in out or "norm.weight" not in out or not any(_LAYER.match(n) for n in out):
        raise ValueError("warm-start expects a Llama-style model exposing model.embed_tokens, "
                         "model.layers and model.norm")
    return out


def _source_name(role: str, name: str, offset: int) -> str:
    """Pretrained tensor name of a bank module's tensor ``name``."""
    if role == "embed" or role == "head":
        return name  # embed_tokens.weight / norm.weight / lm_head.weight
    m = _LAYER.match(name)
    if m is None:
        return name
    return f"layers.{offset + int(m.group(1))}.{m.group(2)}"


@torch.no_grad()
def warm_start_modules(bank: dict[str, nn.Module], topology: PathTopology, source: str | nn.Module) -> None:
    tensors = _pretrained_tensors(load_pretrained(source).eval())
    depth = 1 + max(int(_LAYER.match(n).group(1)) for n in tensors if _LAYER.match(n))
    if depth < topology.total_layers:
        raise ValueError(f"pretrained model has {depth} layers but the path needs {topology.total_layers}")
    for key, module in bank.items():
        role = topology.role_of_key(key)
        offset = 0 if role in ("embed", "head") else topology.offset_of_key(key)
        for name, param in module.named_parameters():
            src = tensors.get(_source_name(role, name, offset))
            if src is None:  # e.g. an untied LM head absent from a model that ties it
                continue
            if src.shape != param.shape:
                raise ValueError(f"{key}.{name}: pretrained shape {tuple(src.shape)} != {tuple(param.shape)}")
            param.copy_(src)
