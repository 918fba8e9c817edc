"""Text -> per-document token tensors (reference ``src/opendipaco/data/text.py``).

Tokenizer libraries are imported lazily so the package imports without them.
"""

from __future__ import annotations

import random
from typing import Iterable

import torch

_HINT = "A HuggingFace tokenizer is required (transformers / tokenizers)."


def load_tokenizer(name: str = "t5-base"):
    try:
        from transformers import AutoTokenizer
    except ImportError as exc:  # pragma: no cover
        raise ImportError(_HINT) from exc
    return AutoTokenizer.from_pretrained(name)


def train_tokenizer(texts: Iterable[str], *, vocab_size: int = 32000, model: str = "unigram",
                    unk_token: str = "<unk>", eos_token: str = "</s>", pad_token: str = "<pad>"):
    """Train a fresh Unigram (SentencePiece-style) or byte-level BPE tokenizer."""
    try:
        from tokenizers import Tokenizer, decoders, models, pre_tokenizers, trainers
        from transformers import PreTrainedTokenizerFast
    except ImportError as exc:  # pragma: no cover
        raise ImportError(_HINT) from exc
    specials = [unk_token, eos_token, pad_token]
    if model == "unigram":
        tok = Tokenizer(models.Unigram())
        tok.pre_tokenizer = pre_tokenizers.Metaspace()
        tok.decoder = decoders.Metaspace()
        trainer = trainers.UnigramTrainer(vocab_size=vocab_size, special_tokens=specials,
                                          unk_token=unk_token)
    elif model == "bpe":
        tok = Tokenizer(models.BPE(unk_token=unk_token))
        tok.pre_tokenizer = pre_tokenizers.ByteLevel()
        tok.decoder = decoders.ByteLevel()
        trainer = trainers.BpeTrainer(vocab_size=vocab_size, special_tokens=specials)
    else:
        raise ValueError(f"model must be 'unigram' or 'bpe', got {model!r}")
    tok.train_from_iterator(texts, trainer)
    return PreTrainedTokenizerFast(tokenizer_object=tok, unk_token=unk_token,
                                   eos_token=eos_token, pad_token=pad_token)


def split_documents(documents, *, val_fraction: float = 0.0, test_fraction: float = 0.0,
                    seed: int = 0):
    """Seeded shuffle, then (train, val, test) split."""
    docs = list(documents)
    random.Random(seed).shuffle(docs)
    n_test, n_val = int(len(docs) * test_fraction), int(len(docs) * val_fraction)
    return docs[n_test + n_val:], docs[n_test:n_test + n_val], docs[:n_test]


def tokenize_one(text: str, tokenizer, *, add_eos: bool = True, max_doc_tokens: int | None = None,
                 min_doc_tokens: int = 1) -> torch.Tensor | None:
    eos = getattr(tokenizer, "eos_token_id", None) if add_eos else None
    ids = list(tokenizer.encode(text, add_special_tokens=False))
    if max_doc_tokens is not None and len(ids) > max_doc_tokens:
        ids = ids[: max_doc_tokens - 1] if eos is not None else ids[:max_doc_tokens]
    if eos is not None:
        ids.append(eos)
    if len(ids) < max(min_doc_tokens, 1):
        return None
    return torch.tensor(ids, dtype=torch.long)


def tokenize_documents(texts: Iterable[str], tokenizer, *, add_eos: bool = True,
                       max_doc_tokens: int | None = None, min_doc_tokens: int = 1):
    out = []
    for t in texts:
        d = tokenize_one(t, tokenizer, add_eos=add_eos, max_doc_tokens=max_doc_tokens,
                         min_doc_tokens=min_doc_tokens)
        if d is not None:
            out.append(d)
    return out
