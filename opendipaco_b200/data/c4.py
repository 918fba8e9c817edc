"""C4 (allenai/c4, English) as tokenized documents.

The dataset is streamed with the Hugging Face ``datasets`` package, imported only when
C4 is actually read (it is not installed on offline machines; every other part of the
package works without it). A tokenized prefix of a split can be cached in one file
(``torch.save`` of the document list, written atomically) so later runs skip the
download. Reference behaviour: ``src/opendipaco/data/c4.py``.
"""

from __future__ import annotations

import itertools
import os
from pathlib import Path

import torch

from .text import load_tokenizer, tokenize_documents

DATASETS_HINT = "The 'datasets' package is required to stream C4 (not installed offline)."


def c4_stream(split: str = "train"):
    """The raw C4 English rows of ``split`` as a streaming iterable (dicts with "text")."""
    try:
        from datasets import load_dataset
    except ImportError as exc:
        raise ImportError(DATASETS_HINT) from exc
    return load_dataset("allenai/c4", "en", split=split, streaming=True)


def save_documents(documents: list[torch.Tensor], path) -> None:
    """Write a document list atomically (a crash leaves the old file or none)."""
    target = Path(path)
    target.parent.mkdir(parents=True, exist_ok=True)
    partial = target.parent / (target.name + ".tmp")
    torch.save(list(documents), partial)
    os.replace(partial, target)


def load_documents(path) -> list[torch.Tensor]:
    return torch.load(path, weights_only=True)


def load_c4_documents(*, split: str = "train", num_documents: int = 10_000, tokenizer=None,
                      tokenizer_name: str = "t5-base", streaming: bool = True,
                      max_doc_tokens: int | None = None, min_doc_tokens: int = 1,
                      add_eos: bool = True, cache_path=None) -> list[torch.Tensor]:
    """The first ``num_documents`` rows of ``split`` tokenized (rows shorter than
    ``min_doc_tokens`` tokens are dropped, so fewer documents may come back). With
    ``cache_path`` an existing cache is returned as it is, or a new one is written."""
    if cache_path is not None and Path(cache_path).exists():
        return load_documents(cache_path)
    if streaming:
        rows = c4_stream(split)
    else:
        try:
            from datasets import load_dataset
        except ImportError as exc:
            raise ImportError(DATASETS_HINT) from exc
        rows = load_dataset("allenai/c4", "en", split=split)
    texts = (row["text"] for row in itertools.islice(rows, num_documents))
    docs = tokenize_documents(texts, tokenizer or load_tokenizer(tokenizer_name), add_eos=add_eos,
                              max_doc_tokens=max_doc_tokens, min_doc_tokens=min_doc_tokens)
    if cache_path is not None:
        save_documents(docs, cache_path)
    return docs
