"""Synthetic token corpora (no network on the training boxes).

* :func:`zipf_documents` -- documents whose token ids follow a Zipf(s) law over the
  vocabulary and whose lengths are uniform in ``[min_len, max_len]``; the
  benchmark workloads use ``s = 1.1``. A per-document random permutation offset
  ("topic") shifts the rank->id map so k-means routing has structure to find.
* :func:`synthetic_documents` lives in :mod:`.spec` (topic-banded uniform ids,
  the reference's generator, kept for spec determinism).

Generation is vectorised with numpy's PCG64 seeded by ``seed`` so the same call
yields byte-identical documents on every rank.
"""

from __future__ import annotations

import numpy as np
import torch


def zipf_documents(*, vocab_size: int, num_documents: int, min_len: int, max_len: int,
                   exponent: float = 1.1, topics: int = 16, seed: int = 0) -> list[torch.Tensor]:
    rng = np.random.Generator(np.random.PCG64(seed))
    ranks = np.arange(1, vocab_size + 1, dtype=np.float64)
    p = ranks ** (-exponent)
    cdf = np.cumsum(p / p.sum())
    lengths = rng.integers(min_len, max_len + 1, size=num_documents)
    topic = rng.integers(0, max(topics, 1), size=num_documents)
    shift = (np.arange(max(topics, 1)) * (vocab_size // max(topics, 1))).astype(np.int64)
    total = int(lengths.sum())
    u = rng.random(total)
    ids = np.searchsorted(cdf, u, side="right").clip(0, vocab_size - 1)
    docs, off = [], 0
    for i, n in enumerate(lengths.tolist()):
        d = (ids[off:off + n] + shift[topic[i]]) % vocab_size
        docs.append(torch.from_numpy(d.astype(np.int64)))
        off += n
    return docs
