"""Learned prefix featurizers (reference ``src/opendipaco/routing/featurizers.py``).

* ``EmbeddingFeaturizer`` -- masked mean/last pooling of a frozen embedding table.
* ``ModelFeaturizer`` -- the paper's ``z``: run prefixes through a reference path of
  the DiPaCo bank (aliased, no copy) and pool the final-norm hidden states.
* ``HFEncoderFeaturizer`` -- pooling of a frozen HuggingFace model's hidden states.

Inputs are right-padded; with causal attention real-token states do not see the
padding, and pooling masks the padded positions out.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn


def _pad_batch(prefixes: list[torch.Tensor], pad_id: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    lens = [int(p.numel()) for p in prefixes]
    width = max(max(lens, default=0), 1)
    ids = torch.full((len(prefixes), width), pad_id, dtype=torch.long)
    mask = torch.zeros((len(prefixes), width), dtype=torch.bool)
    for i, p in enumerate(prefixes):
        if lens[i]:
            ids[i, : lens[i]] = p.to(torch.long)
            mask[i, : lens[i]] = True
    return ids.to(device), mask.to(device)


def _pool(hidden: torch.Tensor, mask: torch.Tensor, pooling: str) -> torch.Tensor:
    if pooling == "mean":
        m = mask.unsqueeze(-1).to(hidden.dtype)
        return (hidden * m).sum(dim=1) / m.sum(dim=1).clamp(min=1.0)
    if pooling == "last":
        last = mask.float().cumsum(dim=1).argmax(dim=1)
        return hidden[torch.arange(hidden.size(0), device=hidden.device), last]
    raise ValueError(f"unknown pooling {pooling!r} (use 'mean' or 'last')")


class EmbeddingFeaturizer:
    def __init__(self, embedding: nn.Embedding | torch.Tensor, *, pooling: str = "mean",
                 normalize: bool = True, pad_id: int = 0, device="cpu", batch_size: int = 256):
        w = embedding.weight if isinstance(embedding, nn.Embedding) else embedding
        self.weight = w.detach().to(device)
        self.feature_dim = self.weight.size(-1)
        self.pooling, self.normalize, self.pad_id = pooling, normalize, pad_id
        self.device, self.batch_size = torch.device(device), batch_size

    @torch.no_grad()
    def __call__(self, prefixes: list[torch.Tensor]) -> torch.Tensor:
        out = []
        for i in range(0, len(prefixes), self.batch_size):
            ids, mask = _pad_batch(prefixes[i:i + self.batch_size], self.pad_id, self.device)
            out.append(_pool(F.embedding(ids, self.weight), mask, self.pooling).cpu())
        feats = torch.cat(out) if out else torch.zeros(0, self.feature_dim)
        return F.normalize(feats, dim=-1) if self.normalize else feats


class ModelFeaturizer:
    def __init__(self, bank: dict[str, nn.Module], config, reference_path=None,
                 pooling: str = "mean", normalize: bool = True, pad_id: int = 0,
                 device="cpu", batch_size: int = 64):
        from ..models.path import build_path_model

        topo = config.build_topology()
        if reference_path is None:
            reference_path = topo.path_from_index(0)
        self.model = build_path_model(config, reference_path, bank, deepcopy=False).to(device)
        self.feature_dim = config.backbone.hidden_size
        self.pooling, self.normalize, self.pad_id = pooling, normalize, pad_id
        self.device, self.batch_size = torch.device(device), batch_size

    @torch.no_grad()
    def __call__(self, prefixes: list[torch.Tensor]) -> torch.Tensor:
        out = []
        for i in range(0, len(prefixes), self.batch_size):
            ids, mask = _pad_batch(prefixes[i:i + self.batch_size], self.pad_id, self.device)
            hidden = self.model.encode(ids)
            out.append(_pool(hidden.float(), mask, self.pooling).cpu())
        feats = torch.cat(out) if out else torch.zeros(0, self.feature_dim)
        return F.normalize(feats, dim=-1) if self.normalize else feats


class HFEncoderFeaturizer:
    def __init__(self, model: str | nn.Module, *, pooling: str = "mean", normalize: bool = True,
                 pad_id: int = 0, device="cpu", batch_size: int = 64):
        if isinstance(model, str):
            from transformers import AutoModel

            model = AutoModel.from_pretrained(model)
        self.model = model.to(device).eval().requires_grad_(False)
        cfg = getattr(model, "config", None)
        self.feature_dim = getattr(cfg, "hidden_size", None)
        pid = getattr(cfg, "pad_token_id", None)
        self.pad_id = pad_id if pid is None else pid
        self.pooling, self.normalize = pooling, normalize
        self.device, self.batch_size = torch.device(device), batch_size

    @staticmethod
    def _hidden(outputs) -> torch.Tensor:
        if torch.is_tensor(outputs):
            return outputs
        return outputs.last_hidden_state if hasattr(outputs, "last_hidden_state") else outputs[0]

    @torch.no_grad()
    def __call__(self, prefixes: list[torch.Tensor]) -> torch.Tensor:
        out = []
        for i in range(0, len(prefixes), self.batch_size):
            ids, mask = _pad_batch(prefixes[i:i + self.batch_size], self.pad_id, self.device)
            h = self._hidden(self.model(input_ids=ids, attention_mask=mask.long()))
            pooled = _pool(h, mask, self.pooling).float().cpu()
            if self.feature_dim is None:
                self.feature_dim = pooled.size(-1)
            out.append(pooled)
        feats = torch.cat(out) if out else torch.zeros(0, self.feature_dim or 1)
        return F.normalize(feats, dim=-1) if self.normalize else feats
