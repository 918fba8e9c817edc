"""Per-path shards: route documents, group them by path, pack into sequences.

Reference: ``src/opendipaco/data/sharding.py:20-198``. ``ShardedCorpus`` keeps the
reference's field names because the object is pickled into a checkpoint's
``corpus.pt`` (loaded with ``weights_only=True`` and an allow-list).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from ..routing.base import Featurizer, Router


def assign_paths(documents: list[torch.Tensor], router: Router, featurizer: Featurizer,
                 prefix_len: int = 32, batch_size: int = 256, top_k: int = 1) -> torch.Tensor:
    """``[N]`` path per document (``top_k == 1``) or ``[N, top_k]`` best paths."""
    if top_k > 1 and not hasattr(router, "predict_topk"):
        raise ValueError("router must implement predict_topk for top_k > 1")
    parts = []
    for i in range(0, len(documents), batch_size):
        feats = featurizer([d[:prefix_len] for d in documents[i:i + batch_size]])
        parts.append((router.predict(feats) if top_k == 1
                      else router.predict_topk(feats, top_k)).cpu())
    if not parts:
        return torch.zeros((0,) if top_k == 1 else (0, top_k), dtype=torch.long)
    return torch.cat(parts)


def pack_sequences(documents: list[torch.Tensor], seq_len: int) -> torch.Tensor:
    """Concatenate and cut into ``[N, seq_len]`` (tail dropped)."""
    if not documents:
        return torch.zeros(0, seq_len, dtype=torch.long)
    flat = torch.cat([d.reshape(-1) for d in documents])
    n = flat.numel() // seq_len
    return flat[: n * seq_len].reshape(n, seq_len) if n else torch.zeros(0, seq_len, dtype=torch.long)


def chunk_documents(documents: list[torch.Tensor], seq_len: int) -> torch.Tensor:
    """Cut each document separately (a window never spans two documents)."""
    out = []
    for d in documents:
        flat = d.reshape(-1)
        n = flat.numel() // seq_len
        if n:
            out.append(flat[: n * seq_len].reshape(n, seq_len))
    return torch.cat(out) if out else torch.zeros(0, seq_len, dtype=torch.long)


@dataclass
class ShardedCorpus:
    """Per-path packed sequences plus the document / token counts behind them."""

    sequences: dict[int, torch.Tensor]
    doc_counts: dict[int, int]
    num_paths: int
    seq_len: int
    token_counts: dict[int, int] | None = None
    val_sequences: dict[int, torch.Tensor] | None = None

    @classmethod
    def from_assignments(cls, documents: list[torch.Tensor], assignments: torch.Tensor,
                         num_paths: int, seq_len: int, val_fraction: float = 0.0,
                         seed: int = 0, pack_mode: str = "pack") -> "ShardedCorpus":
        if pack_mode not in ("pack", "document"):
            raise ValueError(f"pack_mode must be 'pack' or 'document', got {pack_mode!r}")
        to_seq = pack_sequences if pack_mode == "pack" else chunk_documents
        buckets: dict[int, list[torch.Tensor]] = {p: [] for p in range(num_paths)}
        for doc, a in zip(documents, assignments):
            for p in (a.tolist() if a.ndim > 0 else [int(a)]):
                buckets[p].append(doc)
        doc_counts = {p: len(v) for p, v in buckets.items()}
        token_counts = {p: sum(int(d.numel()) for d in v) for p, v in buckets.items()}
        gen = torch.Generator().manual_seed(seed)
        seqs, vals = {}, {}
        for p, docs in buckets.items():
            packed = to_seq(docs, seq_len)
            if val_fraction > 0 and packed.size(0) > 1:
                n_val = max(1, int(packed.size(0) * val_fraction))
                perm = torch.randperm(packed.size(0), generator=gen)
                vals[p], seqs[p] = packed[perm[:n_val]], packed[perm[n_val:]]
            else:
                seqs[p], vals[p] = packed, packed[:0]
        return cls(seqs, doc_counts, num_paths, seq_len, token_counts,
                   vals if val_fraction > 0 else None)

    @classmethod
    def from_documents(cls, documents: list[torch.Tensor], router: Router,
                       featurizer: Featurizer, num_paths: int, seq_len: int,
                       prefix_len: int = 32, top_k: int = 1, val_fraction: float = 0.0,
                       seed: int = 0, pack_mode: str = "pack") -> "ShardedCorpus":
        a = assign_paths(documents, router, featurizer, prefix_len, top_k=top_k)
        return cls.from_assignments(documents, a, num_paths, seq_len, val_fraction, seed, pack_mode)

    def shard(self, path_index: int) -> torch.Tensor:
        return self.sequences[path_index]

    @property
    def has_validation(self) -> bool:
        return self.val_sequences is not None

    def val_shard(self, path_index: int) -> torch.Tensor | None:
        return None if self.val_sequences is None else self.val_sequences.get(path_index)

    def num_sequences(self, path_index: int) -> int:
        return self.sequences[path_index].size(0)

    def shard_weight(self, path_index: int) -> float:
        """alpha_i = tokens_i / total tokens (sequence counts if tokens missing)."""
        if self.token_counts is not None:
            return self.token_counts[path_index] / max(sum(self.token_counts.values()), 1)
        tot = sum(s.size(0) for s in self.sequences.values())
        return self.sequences[path_index].size(0) / max(tot, 1)
