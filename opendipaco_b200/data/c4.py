"""C4 loader (reference ``src/opendipaco/data/c4.py``); network-dependent parts are lazy."""

from __future__ import annotations

import os
from pathlib import Path

import torch

from .text import load_tokenizer, tokenize_documents

DATASETS_HINT = "The 'datasets' package is required to stream C4 (not installed offline)."


def save_documents(documents: list[torch.Tensor], path) -> None:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_suffix(path.suffix + ".tmp")
    torch.save(documents, tmp)
    os.replace(tmp, path)


def load_documents(path) -> list[torch.Tensor]:
    return torch.load(path, weights_only=True)


def load_c4_documents(*, split: str = "train", num_documents: int = 10_000, tokenizer=None,
                      tokenizer_name: str = "t5-base", streaming: bool = True,
                      max_doc_tokens: int | None = None, min_doc_tokens: int = 1,
                      add_eos: bool = True, cache_path=None) -> list[torch.Tensor]:
    if cache_path is not None and Path(cache_path).exists():
        return load_documents(cache_path)
    try:
        from datasets import load_dataset
    except ImportError as exc:
        raise ImportError(DATASETS_HINT) from exc
    tokenizer = tokenizer or load_tokenizer(tokenizer_name)
    ds = load_dataset("allenai/c4", "en", split=split, streaming=streaming)

    def texts():
        for i, row in enumerate(ds):
            if i >= num_documents:
                return
            yield row["text"]

    docs = tokenize_documents(texts(), tokenizer, add_eos=add_eos, max_doc_tokens=max_doc_tokens,
                              min_doc_tokens=min_doc_tokens)
    if cache_path is not None:
        save_documents(docs, cache_path)
    return docs
