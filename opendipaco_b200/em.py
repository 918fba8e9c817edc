"""EM re-sharding (reference ``src/opendipaco/em.py:36-133``).

E-step: score every document under each candidate path (masked mean next-token CE
per document; non-candidates stay ``+inf``) and reassign each document to its
lowest-loss path (or top-k for overlapping shards). ``fit_discriminative_router``
labels held-out documents by their best path and trains the test-time router.

On CUDA, each candidate path's documents are scored with the sm_100a forward and
the fused per-row log-softmax kernel (no fp32 [tokens, vocab] copy).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from .config import DiPaCoConfig
from .data.sharding import ShardedCorpus
from .inference import compose_path
from .routing.base import Featurizer
from .routing.discriminative import DiscriminativeRouter
from .routing.featurizers import _pad_batch


def _token_ce(pred: torch.Tensor, tgt: torch.Tensor) -> torch.Tensor:
    if pred.is_cuda:
        from .ops import loss as L

        return L.cross_entropy_rows(pred.reshape(-1, pred.size(-1)), tgt.reshape(-1)).view(tgt.shape)
    return F.cross_entropy(pred.reshape(-1, pred.size(-1)), tgt.reshape(-1),
                           reduction="none").reshape(tgt.shape)


@torch.no_grad()
def path_losses(documents: list[torch.Tensor], config: DiPaCoConfig, bank: dict[str, nn.Module],
                seq_len: int, candidates: list[int] | None = None, batch_size: int = 16,
                pad_id: int = 0) -> torch.Tensor:
    topo = config.build_topology()
    if candidates is None:
        candidates = list(range(topo.num_paths))
    dev = next(next(iter(bank.values())).parameters()).device
    docs = [d[:seq_len] for d in documents]
    out = torch.full((len(docs), topo.num_paths), float("inf"))
    for p in candidates:
        model = compose_path(config, bank, topo.path_from_index(p)).eval()
        for i in range(0, len(docs), batch_size):
            ids, mask = _pad_batch(docs[i:i + batch_size], pad_id, dev)
            logits, _ = model(ids)
            ce = _token_ce(logits[:, :-1, :], ids[:, 1:]).float()
            m = mask[:, 1:].float()
            out[i:i + ids.size(0), p] = ((ce * m).sum(1) / m.sum(1).clamp(min=1.0)).cpu()
    return out


def assign_paths_by_loss(documents, config, bank, seq_len, top_k: int = 1, candidates=None,
                         batch_size: int = 16, pad_id: int = 0) -> torch.Tensor:
    losses = path_losses(documents, config, bank, seq_len, candidates, batch_size, pad_id)
    return losses.argmin(dim=1) if top_k == 1 else losses.topk(top_k, largest=False, dim=1).indices


def reshard_by_loss(documents, config, bank, seq_len, top_k: int = 1, candidates=None,
                    batch_size: int = 16, pad_id: int = 0) -> ShardedCorpus:
    a = assign_paths_by_loss(documents, config, bank, seq_len, top_k, candidates, batch_size, pad_id)
    return ShardedCorpus.from_assignments(documents, a, config.num_paths, seq_len)


def fit_discriminative_router(documents, config, bank, featurizer: Featurizer, seq_len: int,
                              prefix_len: int = 32, candidates=None, batch_size: int = 16,
                              **fit_kwargs) -> DiscriminativeRouter:
    labels = assign_paths_by_loss(documents, config, bank, seq_len, top_k=1,
                                  candidates=candidates, batch_size=batch_size)
    feats = featurizer([d[:prefix_len] for d in documents])
    router = DiscriminativeRouter(featurizer.feature_dim, config.num_paths)
    router.fit(feats, labels, **fit_kwargs)
    return router
