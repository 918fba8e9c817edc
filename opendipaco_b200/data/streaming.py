"""Sharded, resumable streaming ingestion (reference ``src/opendipaco/data/streaming.py``).

``shard_stream`` partitions a stream round-robin by global index; ``ShardCache``
persists ``(docs, next_index)`` in ONE atomically renamed file
``shard_{id:05d}_of_{n:05d}.pt`` so docs and resume point always agree;
``ingest_c4_shard`` resumes from exactly the next unread index.
"""

from __future__ import annotations

import os
from pathlib import Path

import torch

from .c4 import DATASETS_HINT
from .text import tokenize_one


def _text(item, key: str) -> str:
    return item[key] if isinstance(item, dict) else item


def shard_stream(source, *, num_shards: int, shard_id: int, start_index: int = 0):
    if num_shards < 1 or not 0 <= shard_id < num_shards:
        raise ValueError(f"bad shard {shard_id}/{num_shards}")

    def mine(i):
        return num_shards == 1 or i % num_shards == shard_id

    if start_index and hasattr(source, "skip"):
        for off, item in enumerate(source.skip(start_index)):
            if mine(start_index + off):
                yield start_index + off, item
        return
    for i, item in enumerate(source):
        if i >= start_index and mine(i):
            yield i, item


def stream_documents(source, tokenizer, *, num_shards: int = 1, shard_id: int = 0,
                     start_index: int = 0, limit: int | None = None, text_key: str = "text",
                     add_eos: bool = True, max_doc_tokens: int | None = None,
                     min_doc_tokens: int = 1):
    kept = 0
    for gi, item in shard_stream(source, num_shards=num_shards, shard_id=shard_id,
                                 start_index=start_index):
        doc = tokenize_one(_text(item, text_key), tokenizer, add_eos=add_eos,
                           max_doc_tokens=max_doc_tokens, min_doc_tokens=min_doc_tokens)
        if doc is None:
            continue
        yield gi, doc
        kept += 1
        if limit is not None and kept >= limit:
            return


def c4_stream(split: str):
    try:
        from datasets import load_dataset
    except ImportError as exc:  # pragma: no cover
        raise ImportError(DATASETS_HINT) from exc
    return load_dataset("allenai/c4", "en", split=split, streaming=True)


def stream_c4_documents(*, tokenizer, split: str = "train", num_shards: int = 1, shard_id: int = 0,
                        start_index: int = 0, limit: int | None = None, add_eos: bool = True,
                        max_doc_tokens: int | None = None, min_doc_tokens: int = 1):
    yield from stream_documents(c4_stream(split), tokenizer, num_shards=num_shards,
                                shard_id=shard_id, start_index=start_index, limit=limit,
                                add_eos=add_eos, max_doc_tokens=max_doc_tokens,
                                min_doc_tokens=min_doc_tokens)


class ShardCache:
    """Crash-consistent cache of one ingest shard."""

    def __init__(self, dirpath, *, shard_id: int, num_shards: int):
        if num_shards < 1 or not 0 <= shard_id < num_shards:
            raise ValueError(f"bad shard {shard_id}/{num_shards}")
        self.dir = Path(dirpath)
        self.path = self.dir / f"shard_{shard_id:05d}_of_{num_shards:05d}.pt"

    def load(self) -> tuple[list[torch.Tensor], int]:
        if not self.path.exists():
            return [], 0
        blob = torch.load(self.path, weights_only=True)
        return list(blob["docs"]), int(blob["next_index"])

    def save(self, docs: list[torch.Tensor], next_index: int) -> None:
        self.dir.mkdir(parents=True, exist_ok=True)
        tmp = str(self.path) + ".tmp"
        torch.save({"docs": docs, "next_index": int(next_index), "count": len(docs)}, tmp)
        os.replace(tmp, self.path)


def ingest_c4_shard(cache_dir, *, shard_id: int, num_shards: int, target_docs: int, tokenizer,
                    split: str = "train", flush_every: int = 500, source=None,
                    text_key: str = "text", add_eos: bool = True,
                    max_doc_tokens: int | None = None, min_doc_tokens: int = 1,
                    progress=None) -> list[torch.Tensor]:
    cache = ShardCache(cache_dir, shard_id=shard_id, num_shards=num_shards)
    docs, nxt = cache.load()
    if len(docs) >= target_docs:
        return docs[:target_docs]
    kw = dict(add_eos=add_eos, max_doc_tokens=max_doc_tokens, min_doc_tokens=min_doc_tokens)
    if source is None:
        stream = stream_c4_documents(tokenizer=tokenizer, split=split, num_shards=num_shards,
                                     shard_id=shard_id, start_index=nxt, **kw)
    else:
        stream = stream_documents(source, tokenizer, num_shards=num_shards, shard_id=shard_id,
                                  start_index=nxt, text_key=text_key, **kw)
    pending = 0
    for gi, doc in stream:
        docs.append(doc)
        nxt = gi + 1
        pending += 1
        if pending >= flush_every:
            cache.save(docs, nxt)
            pending = 0
            if progress is not None:
                progress(len(docs), nxt)
        if len(docs) >= target_docs:
            break
    cache.save(docs, nxt)
    if progress is not None:
        progress(len(docs), nxt)
    return docs[:target_docs]
