"""EM re-sharding (reference ``src/opendipaco/em.py:36-133``).

E-step: score every document under each candidate path (masked mean next-token CE
per document; non-candidates stay ``+inf``) and reassign each document to its
lowest-loss path (or top-k for overlapping shards). ``fit_discriminative_router``
labels held-out documents by their best path and trains the test-time router.

On CUDA the candidates are scored side by side: ``GroupedScorer`` runs one grouped
forward for up to 16 candidate paths over each batch of documents (the training
step's grouped tcgen05 kernels, LM head in row chunks, per-row CE kernel), so a batch
costs one set of launches instead of one per path. Shapes the fused kernels do not
take fall back to the module forward path by path.
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
    from .train.scorer import GroupedScorer

    if docs and candidates and GroupedScorer.supported(config, dev):
        return _grouped_path_losses(docs, config, bank, candidates, batch_size, pad_id, dev, out)
    for p in candidates:
        model = compose_path(config, bank, topo.path_from_index(p)).eval()
        for i in range(0, len(docs), batch_size):
            ids, mask = _pad_batch(docs[i:i + batch_size], pad_id, dev)
            logits, _ = model(ids)
            ce = _token_ce(logits[:, :-1, :], ids[:, 1:]).float()
            m = mask[:, 1:].float()
            out[i:i + ids.size(0), p] = ((ce * m).sum(1) / m.sum(1).clamp(min=1.0)).cpu()
    return out


def _grouped_path_losses(docs, config, bank, candidates, batch_size, pad_id, dev, out):
    from .train.scorer import GroupedScorer, group_count, padded_len, shifted_targets

    topo = config.build_topology()
    G = group_count(config, bank, min(16, len(candidates)))
    S = padded_len(max(max(int(d.numel()) for d in docs), 2))
    B = min(batch_size, len(docs))
    sc = GroupedScorer(config, bank, dev, G, B, S)
    for c0 in range(0, len(candidates), G):
        cands = candidates[c0:c0 + G]
        for g in range(G):  # a short last wave repeats its first path in the spare groups
            sc.load(g, topo.path_from_index(cands[g] if g < len(cands) else cands[0]))
        for i in range(0, len(docs), B):
            part = docs[i:i + B]
            ids, mask = _pad_batch(part + [part[0][:0]] * (B - len(part)), pad_id, dev)
            ids = torch.nn.functional.pad(ids, (0, S - ids.size(1)), value=pad_id)
            mask = torch.nn.functional.pad(mask, (0, S - mask.size(1)), value=False)
            tgt = shifted_targets(ids, mask)
            ce = sc.token_losses(ids.expand(G, B, S), tgt.expand(G, B, S))
            m = mask[:, 1:].float().sum(1).clamp(min=1.0)
            loss = (ce.sum(2) / m).cpu()
            for g, p in enumerate(cands):
                out[i:i + len(part), p] = loss[g, :len(part)]
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
