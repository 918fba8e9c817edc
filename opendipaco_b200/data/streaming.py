"""Resumable, sharded ingestion of a document stream.

Several ingest workers split one stream round-robin by the global position of each item
(worker ``shard_id`` of ``num_shards`` takes the items whose index is ``shard_id`` modulo
``num_shards``), so together they read every item exactly once and any of them can stop
and resume independently. A worker keeps its tokenized documents AND the index of the
next unread item in one file, replaced atomically on every flush, so the two can never
disagree after a crash: resuming continues exactly where the last flush left off.

File name and content are shared with the reference (``src/opendipaco/data/
streaming.py``), so a cache written by either framework resumes in the other:
``shard_{id:05d}_of_{n:05d}.pt`` holding ``{"docs": [...], "next_index": int, "count": int}``.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from pathlib import Path

import torch

from .c4 import c4_stream
from .text import tokenize_one


@dataclass(frozen=True)
class Partition:
    """Worker ``shard_id`` of ``num_shards`` round-robin readers of one stream."""

    num_shards: int
    shard_id: int

    def __post_init__(self):
        if self.num_shards < 1 or not 0 <= self.shard_id < self.num_shards:
            raise ValueError(f"bad shard {self.shard_id}/{self.num_shards}")

    def owns(self, index: int) -> bool:
        return index % self.num_shards == self.shard_id


def _positions(source, start: int):
    """(global index, item) from ``start`` on; a source with ``skip`` (a streaming
    dataset) skips the prefix server-side instead of reading it."""
    if start and hasattr(source, "skip"):
        return enumerate(source.skip(start), start)
    return ((i, item) for i, item in enumerate(source) if i >= start)


def shard_stream(source, *, num_shards: int, shard_id: int, start_index: int = 0):
    """This worker's ``(global index, item)`` pairs from ``start_index`` on."""
    part = Partition(num_shards, shard_id)
    return ((i, item) for i, item in _positions(source, start_index) if part.owns(i))


def stream_documents(source, tokenizer, *, num_shards: int = 1, shard_id: int = 0,
                     start_index: int = 0, limit: int | None = None, text_key: str = "text",
                     add_eos: bool = True, max_doc_tokens: int | None = None,
                     min_doc_tokens: int = 1):
    """Tokenized ``(global index, document)`` pairs of this worker's items (items that
    tokenize to fewer than ``min_doc_tokens`` tokens are skipped); at most ``limit``."""
    if limit is not None and limit <= 0:
        return
    produced = 0
    for index, item in shard_stream(source, num_shards=num_shards, shard_id=shard_id, start_index=start_index):
        text = item[text_key] if isinstance(item, dict) else item
        doc = tokenize_one(text, tokenizer, add_eos=add_eos, max_doc_tokens=max_doc_tokens,
                           min_doc_tokens=min_doc_tokens)
        if doc is None:
            continue
        yield index, doc
        produced += 1
        if limit is not None and produced >= limit:
            return


def stream_c4_documents(*, tokenizer, split: str = "train", num_shards: int = 1, shard_id: int = 0,
                        start_index: int = 0, limit: int | None = None, add_eos: bool = True,
                        max_doc_tokens: int | None = None, min_doc_tokens: int = 1):
    return stream_documents(c4_stream(split), tokenizer, num_shards=num_shards, shard_id=shard_id,
                            start_index=start_index, limit=limit, add_eos=add_eos, max_doc_tokens=max_doc_tokens,
                            min_doc_tokens=min_doc_tokens)


class ShardCache:
    """The crash-consistent file of one ingest worker (documents + resume index)."""

    def __init__(self, dirpath, *, shard_id: int, num_shards: int):
        Partition(num_shards, shard_id)  # validates
        self.dir = Path(dirpath)
        self.path = self.dir / f"shard_{shard_id:05d}_of_{num_shards:05d}.pt"

    def load(self) -> tuple[list[torch.Tensor], int]:
        """(documents so far, next unread global index); empty for a new worker."""
        if not self.path.is_file():
            return [], 0
        state = torch.load(self.path, weights_only=True)
        return list(state["docs"]), int(state["next_index"])

    def save(self, docs: list[torch.Tensor], next_index: int) -> None:
        self.dir.mkdir(parents=True, exist_ok=True)
        partial = self.path.parent / (self.path.name + ".tmp")
        torch.save({"docs": list(docs), "next_index": int(next_index), "count": len(docs)}, partial)
        os.replace(partial, self.path)


def ingest_c4_shard(cache_dir, *, shard_id: int, num_shards: int, target_docs: int, tokenizer,
                    split: str = "train", flush_every: int = 500, source=None,
                    text_key: str = "text", add_eos: bool = True,
                    max_doc_tokens: int | None = None, min_doc_tokens: int = 1,
                    progress=None) -> list[torch.Tensor]:
    """Grow this worker's cache to ``target_docs`` documents (reading C4, or ``source``
    when given), flushing every ``flush_every`` new documents; returns the first
    ``target_docs``. ``progress(count, next_index)`` is called after each flush."""
    cache = ShardCache(cache_dir, shard_id=shard_id, num_shards=num_shards)
    docs, next_index = cache.load()
    if len(docs) < target_docs:
        opts = dict(num_shards=num_shards, shard_id=shard_id, start_index=next_index, add_eos=add_eos,
                    max_doc_tokens=max_doc_tokens, min_doc_tokens=min_doc_tokens)
        stream = (stream_c4_documents(tokenizer=tokenizer, split=split, **opts) if source is None
                  else stream_documents(source, tokenizer, text_key=text_key, **opts))
        unsaved = 0

        def flush():
            cache.save(docs, next_index)
            if progress is not None:
                progress(len(docs), next_index)

        for index, doc in stream:
            docs.append(doc)
            next_index, unsaved = index + 1, unsaved + 1
            if len(docs) >= target_docs:
                break
            if unsaved >= flush_every:
                flush()
                unsaved = 0
        flush()
    return docs[:target_docs]
