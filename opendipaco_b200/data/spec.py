"""Shard specs: ship the recipe of a shard instead of its bytes.

A spec names a document source (synthetic parameters or a slice of C4), the routing
state (k-means centroids plus the parameters of the seeded bag-of-tokens featurizer, or
plain round-robin) and how the kept documents are packed. A worker given a spec and its
path index regenerates or streams the documents, routes them with the shipped router,
keeps its own path's and packs them -- the same tensor the server would have sent. The
server only keeps a :class:`SpecCorpus` (the spec plus per-path token counts).

Contracts shared with the reference (``src/opendipaco/data/spec.py``), so a spec made
by either framework materializes to the same bytes in the other:

* the spec dict ``{version, source, routing, num_paths, seq_len, pack_mode, prefix_len}``
  and its source / routing sub-dicts;
* the synthetic documents (topic t draws uniform ids from [t span, (t + 1) span) with
  one torch generator seeded by ``seed``, topics in order);
* routing: k-means ``predict`` over the featurized first ``prefix_len`` tokens, or the
  document's position modulo the path count;
* ``spec_fingerprint`` (sha256 of sorted compact JSON, tensors as the sha256 of their
  bytes, first 16 hex digits) and the cache file ``spec_{fp}_path{idx:04d}.pt``.
"""

from __future__ import annotations

import hashlib
import itertools
import json
import os
from pathlib import Path

import torch

from ..routing.base import BagOfTokensFeaturizer
from ..routing.kmeans import KMeansRouter
from .sharding import chunk_documents, pack_sequences
from .text import tokenize_one

SPEC_VERSION = 1
ROUTE_BATCH = 256  # documents featurized and routed per batch (the result does not depend on it)
PACKERS = {"pack": pack_sequences, "document": chunk_documents}


# ------------------------------------------------------------------ sources
def synthetic_documents(*, vocab_size: int, num_documents: int, doc_len: int, topics: int,
                        seed: int) -> list[torch.Tensor]:
    """``num_documents // topics`` documents per topic, topic t's ids uniform in its
    vocabulary band ``[t span, min((t + 1) span, vocab_size))``."""
    gen = torch.Generator().manual_seed(seed)
    span, per_topic = max(1, vocab_size // topics), max(1, num_documents // topics)
    bands = [(t * span, min((t + 1) * span, vocab_size)) for t in range(topics)]
    return [torch.randint(lo, hi, (doc_len,), generator=gen) for lo, hi in bands for _ in range(per_topic)]


def synthetic_source(*, vocab_size: int, num_documents: int, doc_len: int, topics: int, seed: int) -> dict:
    return {"kind": "synthetic", "vocab_size": vocab_size, "num_documents": num_documents, "doc_len": doc_len,
            "topics": topics, "seed": seed}


def c4_source(*, num_documents: int, tokenizer: str, split: str = "train", max_doc_tokens: int | None = None,
              min_doc_tokens: int = 1, add_eos: bool = True) -> dict:
    return {"kind": "c4", "num_documents": num_documents, "tokenizer": tokenizer, "split": split,
            "max_doc_tokens": max_doc_tokens, "min_doc_tokens": min_doc_tokens, "add_eos": add_eos}


def _synthetic_stream(src: dict, source, tokenizer):
    return iter(synthetic_documents(vocab_size=src["vocab_size"], num_documents=src["num_documents"],
                                    doc_len=src["doc_len"], topics=src["topics"], seed=src["seed"]))


def _c4_stream(src: dict, source, tokenizer):
    if source is None:
        from .c4 import c4_stream

        source = c4_stream(src["split"])
    if tokenizer is None:
        from .text import load_tokenizer

        tokenizer = load_tokenizer(src["tokenizer"])
    for item in itertools.islice(source, src["num_documents"]):
        doc = tokenize_one(item["text"] if isinstance(item, dict) else item, tokenizer, add_eos=src["add_eos"],
                           max_doc_tokens=src["max_doc_tokens"], min_doc_tokens=src["min_doc_tokens"])
        if doc is not None:
            yield doc


_SOURCES = {"synthetic": _synthetic_stream, "c4": _c4_stream}


def iter_spec_documents(spec: dict, *, source=None, tokenizer=None):
    """The documents of the spec's source, in order (``source`` / ``tokenizer`` override
    the C4 stream and tokenizer the spec names, e.g. for offline tests)."""
    src = spec["source"]
    stream = _SOURCES.get(src["kind"])
    if stream is None:
        raise ValueError(f"unknown source kind {src['kind']!r}")
    return stream(src, source, tokenizer)


# ------------------------------------------------------------------ routing
def round_robin_routing() -> dict:
    return {"kind": "round_robin"}


def kmeans_routing(centroids: torch.Tensor, *, vocab_size: int, feature_dim: int, seed: int = 0) -> dict:
    return {"kind": "kmeans", "centroids": centroids.detach().cpu(),
            "featurizer": {"kind": "bag_of_tokens", "vocab_size": vocab_size, "feature_dim": feature_dim,
                           "seed": seed}}


def fit_routing_from_source(source: dict, *, num_paths: int, vocab_size: int, seq_len: int, sample: int,
                            feature_dim: int, router_seed: int = 0, feat_seed: int = 0, doc_source=None,
                            tokenizer=None) -> dict:
    """k-means routing fitted on the first ``seq_len`` tokens of the first ``sample``
    documents (round-robin when there are fewer documents than paths); the fit's
    parameters are recorded so any peer can re-fit and check it."""
    if sample < 1:
        raise ValueError(f"router sample must be >= 1, got {sample}")
    docs = itertools.islice(iter_spec_documents({"source": source}, source=doc_source, tokenizer=tokenizer), sample)
    prefixes = [d[:seq_len] for d in docs]
    if len(prefixes) < num_paths:
        return round_robin_routing()
    featurize = BagOfTokensFeaturizer(vocab_size, feature_dim=feature_dim, seed=feat_seed)
    router = KMeansRouter(num_paths, seed=router_seed).fit(featurize(prefixes))
    return {**kmeans_routing(router.centroids, vocab_size=vocab_size, feature_dim=feature_dim, seed=feat_seed),
            "fit": {"sample": sample, "router_seed": router_seed}}


def verify_routing(spec: dict, *, source=None, tokenizer=None, atol: float = 1e-3, rtol: float = 1e-3) -> bool:
    """Re-fit the spec's router from its declared source and compare the centroids: a
    worker refuses a router that does not reproduce (it could route data adversarially)."""
    routing = spec["routing"]
    if routing.get("kind") == "round_robin":
        return True
    if routing.get("kind") != "kmeans":
        raise ValueError(f"cannot verify routing kind {routing.get('kind')!r}")
    fit, feat = routing.get("fit"), routing["featurizer"]
    if not fit:
        raise ValueError("spec has no reproducible fit metadata; verification needs a sampled fit")
    if feat.get("kind") != "bag_of_tokens":
        raise ValueError(f"cannot verify featurizer kind {feat.get('kind')!r}")
    refit = fit_routing_from_source(spec["source"], num_paths=spec["num_paths"], vocab_size=feat["vocab_size"],
                                    seq_len=spec["seq_len"], sample=fit["sample"], feature_dim=feat["feature_dim"],
                                    router_seed=fit["router_seed"], feat_seed=feat.get("seed", 0),
                                    doc_source=source, tokenizer=tokenizer)
    if refit.get("kind") != "kmeans":
        raise ValueError("could not reproduce a k-means fit from the current source")
    shipped, again = routing["centroids"].float(), refit["centroids"].float()
    return shipped.shape == again.shape and torch.allclose(shipped, again, atol=atol, rtol=rtol)


def _route_batch_fn(spec: dict):
    """``fn(start, docs) -> path per document`` for the spec's routing."""
    routing, paths = spec["routing"], spec["num_paths"]
    if routing["kind"] == "round_robin":
        return lambda start, docs: [(start + i) % paths for i in range(len(docs))]
    if routing["kind"] != "kmeans":
        raise ValueError(f"unknown routing kind {routing['kind']!r}")
    f = routing["featurizer"]
    if f["kind"] != "bag_of_tokens":
        raise ValueError(f"unknown featurizer kind {f['kind']!r}")
    featurize = BagOfTokensFeaturizer(f["vocab_size"], feature_dim=f["feature_dim"], seed=f["seed"])
    router = KMeansRouter(paths)
    router.centroids = routing["centroids"]
    plen = spec["prefix_len"]
    return lambda start, docs: router.predict(featurize([d[:plen] for d in docs])).tolist()


def iter_assignments(spec: dict, docs, *, source=None, tokenizer=None):
    """``(document, path)`` for every document (the spec's own documents when ``docs``
    is None)."""
    if docs is None:
        docs = iter_spec_documents(spec, source=source, tokenizer=tokenizer)
    route, start = _route_batch_fn(spec), 0
    for batch in itertools.batched(docs, ROUTE_BATCH):
        yield from zip(batch, route(start, batch))
        start += len(batch)


# ------------------------------------------------------------------ specs
def make_shard_spec(*, source: dict, routing: dict, num_paths: int, seq_len: int, pack_mode: str = "pack",
                    prefix_len: int = 32) -> dict:
    if pack_mode not in PACKERS:
        raise ValueError(f"pack_mode must be 'pack' or 'document', got {pack_mode!r}")
    return {"version": SPEC_VERSION, "source": source, "routing": routing, "num_paths": num_paths,
            "seq_len": seq_len, "pack_mode": pack_mode, "prefix_len": prefix_len}


def _tensor_digest(obj):
    if torch.is_tensor(obj):
        raw = obj.detach().cpu().contiguous().reshape(-1).view(torch.uint8).numpy().tobytes()
        return {"$tensor": hashlib.sha256(raw).hexdigest()}
    raise TypeError(f"spec values must be JSON data or tensors, got {type(obj)}")


def spec_fingerprint(spec: dict) -> str:
    text = json.dumps(spec, sort_keys=True, separators=(",", ":"), default=_tensor_digest)
    return hashlib.sha256(text.encode()).hexdigest()[:16]


def materialize_shard(spec: dict, path_index: int, *, source=None, tokenizer=None, cache_dir=None) -> torch.Tensor:
    """Path ``path_index``'s shard, built from the spec (and cached in ``cache_dir``)."""
    if not 0 <= path_index < spec["num_paths"]:
        raise ValueError(f"bad path_index {path_index} for {spec['num_paths']} paths")
    cached = None
    if cache_dir is not None:
        cached = Path(cache_dir) / f"spec_{spec_fingerprint(spec)}_path{path_index:04d}.pt"
        if cached.is_file():
            return torch.load(cached, weights_only=True)
    mine = [d for d, p in iter_assignments(spec, None, source=source, tokenizer=tokenizer) if p == path_index]
    shard = PACKERS[spec["pack_mode"]](mine, spec["seq_len"])
    if cached is not None:
        cached.parent.mkdir(parents=True, exist_ok=True)
        partial = cached.parent / (cached.name + ".tmp")
        torch.save(shard, partial)
        os.replace(partial, cached)
    return shard


def _token_counts(spec: dict, assignments) -> dict[int, int]:
    counts = dict.fromkeys(range(spec["num_paths"]), 0)
    for doc, path in assignments:
        counts[path] += int(doc.numel())
    return counts


class SpecCorpus:
    """The server-side corpus in spec mode: the spec and per-path token counts (for the
    outer weights); it holds no shard bytes."""

    def __init__(self, spec: dict, token_counts: dict[int, int]):
        self.spec = spec
        self.token_counts = dict(token_counts)
        self.num_paths = spec["num_paths"]
        self.seq_len = spec["seq_len"]

    @classmethod
    def from_documents(cls, spec: dict, documents) -> "SpecCorpus":
        return cls(spec, _token_counts(spec, iter_assignments(spec, documents)))

    @classmethod
    def build(cls, spec: dict, *, source=None, tokenizer=None) -> "SpecCorpus":
        return cls(spec, _token_counts(spec, iter_assignments(spec, None, source=source, tokenizer=tokenizer)))

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
