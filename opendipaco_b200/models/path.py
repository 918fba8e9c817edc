"""Module bank and single-path models.

Reference: ``src/opendipaco/model.py:25-241``.

* :func:`build_module_bank` builds one authoritative instance of every module key
  (identical-expert init by deep-copying a per-segment template; optional tied
  embed/head; ``seed=`` forks the CPU RNG so the build is a pure function).
* :class:`PathModel` composes embed -> body blocks -> head for one path. Loss is
  the mean next-token cross-entropy (labels shifted by one, ``ignore_index=-100``).
* :func:`build_path_model` deep-copies the selection in one call so tied weights
  stay tied (or aliases the bank with ``deepcopy=False``).

The B200 training executor does not call :meth:`PathModel.forward` in its hot
loop (it drives the kernels directly over flat buffers, see
``opendipaco_b200/train/fused.py``), but this module is the public API and the
CPU oracle, and on CUDA its forward runs on the sm_100a kernels.
"""

from __future__ import annotations

import copy

import torch
import torch.nn.functional as F
from torch import nn
from torch.utils.checkpoint import checkpoint

from ..config import DiPaCoConfig
from ..topology import Path, PathTopology, embed_key, head_key, is_private_key
from .llama import BlockModule, EmbeddingModule, HeadModule, rope_cos_sin


def _build_module(topo: PathTopology, bb, key: str) -> nn.Module:
    role = topo.role_of_key(key)
    if role == "embed":
        return EmbeddingModule(bb)
    if role == "head":
        return HeadModule(bb)
    return BlockModule(bb, topo.layers_of_key(key), topo.offset_of_key(key))


def build_module_bank(config: DiPaCoConfig, *, seed: int | None = None) -> dict[str, nn.Module]:
    """One instance per module key; identical-expert init unless disabled."""
    if seed is not None:
        with torch.random.fork_rng(devices=[]):
            torch.manual_seed(seed)
            return build_module_bank(config)
    bb = config.backbone
    topo = config.build_topology()
    bank: dict[str, nn.Module] = {}
    first: dict[int, nn.Module] = {}
    for key in topo.module_keys():
        seg = topo._segment_index_of_key(key)
        if seg not in first:
            first[seg] = bank[key] = _build_module(topo, bb, key)
        elif config.identical_expert_init:
            bank[key] = copy.deepcopy(first[seg])
        else:
            bank[key] = _build_module(topo, bb, key)
    if config.tie_word_embeddings and embed_key() in bank and head_key() in bank:
        bank[head_key()].lm_head.weight = bank[embed_key()].embed_tokens.weight
    return bank


class PathModel(nn.Module):
    """embed -> body blocks/experts -> head for a single path."""

    def __init__(self, config: DiPaCoConfig, path: Path, modules: dict[str, nn.Module]):
        super().__init__()
        self.config = config
        self.path = path
        self.topology = config.build_topology()
        self.embed: nn.Module | None = None
        self.head: nn.Module | None = None
        self.body = nn.ModuleList()
        self._body_keys: list[str] = []
        self._embed_key = self._head_key = None
        for key in self.topology.path_module_keys(path):
            role = self.topology.role_of_key(key)
            if role == "embed":
                self.embed, self._embed_key = modules[key], key
            elif role == "head":
                self.head, self._head_key = modules[key], key
            else:
                self.body.append(modules[key])
                self._body_keys.append(key)
        if self.embed is None or self.head is None:
            raise ValueError("a path must contain an embedding and a head segment")
        self.checkpoint = False
        self.loss_chunks = 1
        self._rope_cache: dict = {}

    def modules_by_key(self) -> dict[str, nn.Module]:
        out = {self._embed_key: self.embed, self._head_key: self.head}
        out.update(zip(self._body_keys, self.body))
        return out

    def _rope(self, seqlen: int, device) -> tuple[torch.Tensor, torch.Tensor]:
        key = (seqlen, str(device))
        if key not in self._rope_cache:
            bb = self.config.backbone
            self._rope_cache[key] = rope_cos_sin(bb.head_dim, bb.rope_theta, seqlen, device)
        return self._rope_cache[key]

    def _backbone(self, input_ids: torch.Tensor, attention_mask: torch.Tensor | None):
        hidden = self.embed(input_ids)
        cos, sin = self._rope(input_ids.shape[1], input_ids.device)
        pad = attention_mask.bool() if attention_mask is not None else None
        ckpt = self.checkpoint and self.training and torch.is_grad_enabled()
        for block in self.body:
            if ckpt:
                hidden = checkpoint(block, hidden, cos, sin, pad, use_reentrant=False)
            else:
                hidden = block(hidden, cos, sin, pad)
        return hidden

    @torch.no_grad()
    def encode(self, input_ids: torch.Tensor, attention_mask: torch.Tensor | None = None):
        """Final hidden states after the head's norm (routing features ``z``)."""
        hidden = self._backbone(input_ids, attention_mask)
        norm = getattr(self.head, "norm", None)
        return norm(hidden) if norm is not None else hidden

    def _chunked_loss(self, hidden: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        norm = getattr(self.head, "norm", None)
        normed = norm(hidden) if norm is not None else hidden
        h = normed[:, :-1, :].reshape(-1, normed.size(-1))
        y = labels[:, 1:].reshape(-1)
        total = torch.zeros((), dtype=torch.float32, device=h.device)
        count = 0
        for hc, yc in zip(h.chunk(self.loss_chunks), y.chunk(self.loss_chunks)):
            total = total + F.cross_entropy(self.head.lm_head(hc), yc, ignore_index=-100,
                                            reduction="sum").float()
            count += int((yc != -100).sum())
        return total / max(count, 1)

    def forward(self, input_ids: torch.Tensor, attention_mask: torch.Tensor | None = None,
                labels: torch.Tensor | None = None):
        hidden = self._backbone(input_ids, attention_mask)
        if labels is not None and self.loss_chunks > 1:
            return None, self._chunked_loss(hidden, labels)
        logits = self.head(hidden)
        loss = None
        if labels is not None:
            pred = logits[:, :-1, :].reshape(-1, logits.size(-1))
            loss = F.cross_entropy(pred.float() if pred.is_cuda else pred,
                                   labels[:, 1:].reshape(-1), ignore_index=-100)
        return logits, loss


def build_path_model(config: DiPaCoConfig, path: Path, bank: dict[str, nn.Module],
                     deepcopy: bool = True, dedup_private: bool = False) -> PathModel:
    """Compose a path from the bank (deep copy in ONE call so ties survive)."""
    keys = config.build_topology().path_module_keys(path)
    missing = [k for k in keys if k not in bank]
    if missing:
        raise KeyError(
            f"bank is missing modules {missing} needed for path {path}. Building a path "
            "needs the full module bank; under distributed training each rank holds only "
            "its own paths' modules, so gather it first with "
            "opendipaco_b200.gather_full_bank(backend, engine.bank, config)."
        )
    chosen = {k: bank[k] for k in keys}
    if deepcopy:
        if dedup_private:
            shared = copy.deepcopy({k: m for k, m in chosen.items() if not is_private_key(k)})
            chosen = {k: shared.get(k, chosen[k]) for k in keys}
        else:
            chosen = copy.deepcopy(chosen)
    return PathModel(config, path, chosen)
