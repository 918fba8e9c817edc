"""Checkpoint / resume (reference ``src/opendipaco/checkpoint.py:33-138``).

A checkpoint is a directory: ``rank{r}.pt`` per rank (``engine.state_dict()``,
written to ``.pt.tmp`` then ``os.replace``), plus rank 0's ``meta.json`` (format,
fingerprint, world_size, materialize, global_round, total_rounds) and optional
``corpus.pt`` / ``extra.pt``; then a backend barrier. Loads use
``weights_only=True`` with the corpus classes allow-listed. The layout and payload
schema are the reference's, so a run can resume across the two frameworks'
checkpoint readers.
"""

from __future__ import annotations

import json
import os
from pathlib import Path as FsPath

import torch

from .data.sharding import ShardedCorpus
from .data.spec import SpecCorpus

torch.serialization.add_safe_globals([ShardedCorpus, SpecCorpus])

__all__ = ["save_checkpoint", "load_checkpoint", "latest_checkpoint"]


def _rank_of(engine) -> int:
    return int(getattr(engine.backend, "rank", 0))


def _atomic_save(obj, path: FsPath) -> None:
    tmp = path.with_suffix(path.suffix + ".tmp")
    torch.save(obj, tmp)
    os.replace(tmp, path)


def save_checkpoint(engine, dirpath, *, corpus=None, extra=None) -> str:
    d = FsPath(dirpath)
    rank = _rank_of(engine)
    state = engine.state_dict()
    d.mkdir(parents=True, exist_ok=True)
    _atomic_save(state, d / f"rank{rank}.pt")
    if rank == 0:
        meta = {k: state[k] for k in ("format", "fingerprint", "world_size", "materialize",
                                     "global_round", "total_rounds")}
        tmp = d / "meta.json.tmp"
        tmp.write_text(json.dumps(meta, indent=2))
        os.replace(tmp, d / "meta.json")
        if corpus is not None:
            _atomic_save(corpus, d / "corpus.pt")
        if extra is not None:
            _atomic_save(extra, d / "extra.pt")
    engine.backend.barrier()
    return str(d)


def load_checkpoint(engine, dirpath, *, strict: bool = True) -> dict:
    d = FsPath(dirpath)
    rank = _rank_of(engine)
    f = d / f"rank{rank}.pt"
    if not f.exists():
        raise FileNotFoundError(f"no checkpoint shard for rank {rank} at {f}")
    engine.load_state_dict(torch.load(f, map_location="cpu", weights_only=True), strict=strict)
    out = {}
    for name in ("corpus", "extra"):
        p = d / f"{name}.pt"
        if p.exists():
            out[name] = torch.load(p, map_location="cpu", weights_only=True)
    return out


def latest_checkpoint(root) -> str | None:
    root = FsPath(root)
    if not root.is_dir():
        return None
    best = None
    for child in root.iterdir():
        meta = child / "meta.json"
        if not (child.is_dir() and meta.exists()):
            continue
        try:
            rnd = json.loads(meta.read_text()).get("global_round", -1)
        except (ValueError, OSError):
            continue
        if best is None or rnd > best[0]:
            best = (rnd, str(child))
    return best[1] if best else None
