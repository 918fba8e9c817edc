"""Shard specs: ship the recipe for a shard, not its bytes.

Reference: ``src/opendipaco/data/spec.py:45-412``. A spec names a document source
(synthetic parameters or a C4 slice), the routing state (k-means centroids plus
the seeded bag-of-tokens featurizer's parameters, or round-robin) and the packing
parameters. A worker regenerates / streams the documents, routes them with the
shipped router, keeps its own path's, and packs them: same bytes as the server
would have shipped. The server keeps a :class:`SpecCorpus` (spec + per-path token
counts, no sequences).

The spec dict layout (keys ``version, source, routing, num_paths, seq_len,
pack_mode, prefix_len``) and the cache-file name ``spec_{fp}_path{idx:04d}.pt``
are wire/disk formats and are kept as in the reference.
"""

from __future__ import annotations

import hashlib
import json
import os
from pathlib import Path

import torch

from ..routing.base import BagOfTokensFeaturizer
from ..routing.kmeans import KMeansRouter
from .sharding import chunk_documents, pack_sequences
from .text import tokenize_one

SPEC_VERSION = 1
_ASSIGN_BATCH = 256


def synthetic_documents(*, vocab_size: int, num_documents: int, doc_len: int, topics: int,
                        seed: int) -> list[torch.Tensor]:
    """Topic-banded uniform ids: topic t draws from ``[t*span, (t+1)*span)``."""
    g = torch.Generator().manual_seed(seed)
    span = max(1, vocab_size // topics)
    per = max(1, num_documents // topics)
    out = []
    for t in range(topics):
        lo, hi = t * span, min((t + 1) * span, vocab_size)
        out += [torch.randint(lo, hi, (doc_len,), generator=g) for _ in range(per)]
    return out


def synthetic_source(*, vocab_size: int, num_documents: int, doc_len: int, topics: int,
                     seed: int) -> dict:
    return {"kind": "synthetic", "vocab_size": vocab_size, "num_documents": num_documents,
            "doc_len": doc_len, "topics": topics, "seed": seed}


def c4_source(*, num_documents: int, tokenizer: str, split: str = "train",
              max_doc_tokens: int | None = None, min_doc_tokens: int = 1,
              add_eos: bool = True) -> dict:
    return {"kind": "c4", "num_documents": num_documents, "tokenizer": tokenizer, "split": split,
            "max_doc_tokens": max_doc_tokens, "min_doc_tokens": min_doc_tokens, "add_eos": add_eos}


def iter_spec_documents(spec: dict, *, source=None, tokenizer=None):
    src = spec["source"]
    if src["kind"] == "synthetic":
        yield from synthetic_documents(vocab_size=src["vocab_size"],
                                       num_documents=src["num_documents"],
                                       doc_len=src["doc_len"], topics=src["topics"],
                                       seed=src["seed"])
        return
    if src["kind"] != "c4":
        raise ValueError(f"unknown source kind {src['kind']!r}")
    if source is None:
        from .streaming import c4_stream

        source = c4_stream(src["split"])
    if tokenizer is None:
        from .text import load_tokenizer

        tokenizer = load_tokenizer(src["tokenizer"])
    for i, item in enumerate(source):
        if i >= src["num_documents"]:
            return
        doc = tokenize_one(item["text"] if isinstance(item, dict) else item, tokenizer,
                           add_eos=src["add_eos"], max_doc_tokens=src["max_doc_tokens"],
                           min_doc_tokens=src["min_doc_tokens"])
        if doc is not None:
            yield doc


def round_robin_routing() -> dict:
    return {"kind": "round_robin"}


def kmeans_routing(centroids: torch.Tensor, *, vocab_size: int, feature_dim: int,
                   seed: int = 0) -> dict:
    return {"kind": "kmeans", "centroids": centroids.detach().cpu(),
            "featurizer": {"kind": "bag_of_tokens", "vocab_size": vocab_size,
                           "feature_dim": feature_dim, "seed": seed}}


def fit_routing_from_source(source: dict, *, num_paths: int, vocab_size: int, seq_len: int,
                            sample: int, feature_dim: int, router_seed: int = 0,
                            feat_seed: int = 0, doc_source=None, tokenizer=None) -> dict:
    """Fit k-means on the first ``sample`` document prefixes; round-robin if too few."""
    if sample < 1:
        raise ValueError(f"router sample must be >= 1, got {sample}")
    feat = BagOfTokensFeaturizer(vocab_size, feature_dim=feature_dim, seed=feat_seed)
    prefixes = []
    for doc in iter_spec_documents({"source": source}, source=doc_source, tokenizer=tokenizer):
        prefixes.append(doc[:seq_len])
        if len(prefixes) >= sample:
            break
    if len(prefixes) < num_paths:
        return round_robin_routing()
    router = KMeansRouter(num_paths, seed=router_seed).fit(feat(prefixes))
    out = kmeans_routing(router.centroids, vocab_size=vocab_size, feature_dim=feature_dim,
                         seed=feat_seed)
    out["fit"] = {"sample": sample, "router_seed": router_seed}
    return out


def verify_routing(spec: dict, *, source=None, tokenizer=None, atol: float = 1e-3,
                   rtol: float = 1e-3) -> bool:
    """Re-fit from the spec's own source and compare centroids (refuse on mismatch)."""
    routing = spec["routing"]
    kind = routing.get("kind")
    if kind == "round_robin":
        return True
    if kind != "kmeans":
        raise ValueError(f"cannot verify routing kind {kind!r}")
    fit = routing.get("fit")
    if not fit:
        raise ValueError("spec has no reproducible fit metadata; verification needs a sampled fit")
    feat = routing["featurizer"]
    if feat.get("kind") != "bag_of_tokens":
        raise ValueError(f"cannot verify featurizer kind {feat.get('kind')!r}")
    again = fit_routing_from_source(spec["source"], num_paths=spec["num_paths"],
                                    vocab_size=feat["vocab_size"], seq_len=spec["seq_len"],
                                    sample=fit["sample"], feature_dim=feat["feature_dim"],
                                    router_seed=fit["router_seed"], feat_seed=feat.get("seed", 0),
                                    doc_source=source, tokenizer=tokenizer)
    if again.get("kind") != "kmeans":
        raise ValueError("could not reproduce a k-means fit from the current source")
    a, b = routing["centroids"].float(), again["centroids"].float()
    return a.shape == b.shape and torch.allclose(a, b, atol=atol, rtol=rtol)


def _build_predictor(spec: dict):
    routing = spec["routing"]
    if routing["kind"] == "round_robin":
        return None
    if routing["kind"] != "kmeans":
        raise ValueError(f"unknown routing kind {routing['kind']!r}")
    f = routing["featurizer"]
    if f["kind"] != "bag_of_tokens":
        raise ValueError(f"unknown featurizer kind {f['kind']!r}")
    feat = BagOfTokensFeaturizer(f["vocab_size"], feature_dim=f["feature_dim"], seed=f["seed"])
    router = KMeansRouter(spec["num_paths"])
    router.centroids = routing["centroids"]
    return lambda prefixes: router.predict(feat(prefixes))


def iter_assignments(spec: dict, docs, *, source=None, tokenizer=None):
    """Yield ``(doc, path)`` for every document, routed in batches of 256."""
    if docs is None:
        docs = iter_spec_documents(spec, source=source, tokenizer=tokenizer)
    predict = _build_predictor(spec)
    if predict is None:
        for i, d in enumerate(docs):
            yield d, i % spec["num_paths"]
        return
    plen, batch = spec["prefix_len"], []

    def flush(b):
        yield from zip(b, predict([d[:plen] for d in b]).tolist())

    for d in docs:
        batch.append(d)
        if len(batch) >= _ASSIGN_BATCH:
            yield from flush(batch)
            batch = []
    if batch:
        yield from flush(batch)


def make_shard_spec(*, source: dict, routing: dict, num_paths: int, seq_len: int,
                    pack_mode: str = "pack", prefix_len: int = 32) -> dict:
    if pack_mode not in ("pack", "document"):
        raise ValueError(f"pack_mode must be 'pack' or 'document', got {pack_mode!r}")
    return {"version": SPEC_VERSION, "source": source, "routing": routing, "num_paths": num_paths,
            "seq_len": seq_len, "pack_mode": pack_mode, "prefix_len": prefix_len}


def spec_fingerprint(spec: dict) -> str:
    """sha256[:16] of canonical JSON with tensors replaced by the sha256 of their bytes."""
    def canon(o):
        if torch.is_tensor(o):
            raw = o.detach().cpu().contiguous().reshape(-1).view(torch.uint8).numpy().tobytes()
            return {"$tensor": hashlib.sha256(raw).hexdigest()}
        if isinstance(o, dict):
            return {k: canon(v) for k, v in sorted(o.items())}
        if isinstance(o, (list, tuple)):
            return [canon(v) for v in o]
        return o
    blob = json.dumps(canon(spec), sort_keys=True, separators=(",", ":"))
    return hashlib.sha256(blob.encode()).hexdigest()[:16]


def materialize_shard(spec: dict, path_index: int, *, source=None, tokenizer=None,
                      cache_dir=None) -> torch.Tensor:
    if not 0 <= path_index < spec["num_paths"]:
        raise ValueError(f"bad path_index {path_index} for {spec['num_paths']} paths")
    cache = None
    if cache_dir is not None:
        cache = Path(cache_dir) / f"spec_{spec_fingerprint(spec)}_path{path_index:04d}.pt"
        if cache.exists():
            return torch.load(cache, weights_only=True)
    kept = [d for d, p in iter_assignments(spec, None, source=source, tokenizer=tokenizer)
            if p == path_index]
    packed = (pack_sequences if spec["pack_mode"] == "pack" else chunk_documents)(kept, spec["seq_len"])
    if cache is not None:
        cache.parent.mkdir(parents=True, exist_ok=True)
        tmp = str(cache) + ".tmp"
        torch.save(packed, tmp)
        os.replace(tmp, cache)
    return packed


class SpecCorpus:
    """Server-side corpus in spec mode: the spec + per-path token counts only."""

    def __init__(self, spec: dict, token_counts: dict[int, int]):
        self.spec = spec
        self.token_counts = dict(token_counts)
        self.num_paths = spec["num_paths"]
        self.seq_len = spec["seq_len"]

    @classmethod
    def from_documents(cls, spec: dict, documents) -> "SpecCorpus":
        counts = dict.fromkeys(range(spec["num_paths"]), 0)
        for d, p in iter_assignments(spec, documents):
            counts[p] += int(d.numel())
        return cls(spec, counts)

    @classmethod
    def build(cls, spec: dict, *, source=None, tokenizer=None) -> "SpecCorpus":
        counts = dict.fromkeys(range(spec["num_paths"]), 0)
        for d, p in iter_assignments(spec, None, source=source, tokenizer=tokenizer):
            counts[p] += int(d.numel())
        return cls(spec, counts)

    def shard(self, path_index: int) -> torch.Tensor:
        raise RuntimeError("SpecCorpus holds no shard bytes; workers materialize shards "
                           "locally with materialize_shard(spec, path).")

    @property
    def has_validation(self) -> bool:
        return False

    def val_shard(self, path_index: int):
        return None

    def shard_weight(self, path_index: int) -> float:
        return self.token_counts[path_index] / max(sum(self.token_counts.values()), 1)
