"""Dynamics harness: do the asynchronous and compressed variants of DiPaCo still
converge like the synchronous algorithm? Every arm trains the same documents with the
same seed for the same number of generations in one process (loopback TCP for the
cluster arms) and is scored by the same router-free metric: the held-out perplexity
of each document under its best path.

    python -m opendipaco_b200.launch.dynamics --rounds 6 --arms sync,async,int8,int4

Arms (the comparisons of the reference's ``examples/validate_dynamics.py``):

* ``sync``          -- the synchronous engine (sum of sharing paths' pseudo-gradients,
  one outer step per round): the anchor;
* ``async``         -- the sharded scheduler with racing workers (per-contribution outer
  steps, inverse-staleness damping);
* ``int8`` / ``int4`` -- compressed pseudo-gradients on the wire (error feedback);
* ``robust``        -- owner-side quorum buffers and trimmed-mean aggregation;
* ``delta_down``    -- workers rebuild weights from keyframes plus int8 deltas;
* ``sparse_up``     -- the top quarter of each pseudo-gradient row, the rest carried;
* ``adam8bit``      -- blockwise 8-bit inner optimizer moments;
* ``decentralized`` -- no scheduler: self-assigned slots, owner-minted grants, pushes to
  every owner of a key.

What this does not cover: wide-area latency, NAT and real churn (``launch/churn.py``
covers churn on loopback).
"""

from __future__ import annotations

import argparse
import json
import math
import time

import torch

from ..data import synthetic_documents
from ..em import path_losses
from ..models.path import build_module_bank
from ..parallel.backend import LocalBackend
from ..train import DiPaCoEngine
from .config import LaunchConfig, diloco_config, dipaco_config
from .roles import build_server_corpus, run_local

ARMS = {
    "sync": None,
    "async": {},
    "int8": {"transport": {"compress": "int8"}},
    "int4": {"transport": {"compress": "int4"}},
    "robust": {"robustness": {"mode": "on", "quorum_target": 2, "quorum_timeout": 2.0}},
    "delta_down": {"transport": {"down": "delta"}},
    "sparse_up": {"transport": {"up_density": 0.25}},
    "adam8bit": {"diloco": {"optim_8bit": True}},
    "decentralized": {"schedule": {"mode": "decentralized", "read_quorum": 1, "lease_ttl": 5.0},
                      "ownership": {"mode": "rendezvous", "k": 2, "heartbeat_interval": 1.0,
                                    "replicate_interval": 2.0}},
}


def base_config(rounds: int = 6, *, hidden: int = 64, docs: int = 160, workers: int = 3, seed: int = 0) -> dict:
    return {"mode": "sharded",
            "model": {"vocab_size": 128, "hidden_size": hidden, "num_attention_heads": 4,
                      "intermediate_size": 2 * hidden, "max_position_embeddings": 128, "layers_per_level": [1, 1],
                      "level_sizes": [2, 2], "sequence_length": 32},
            "diloco": {"inner_steps": 8, "inner_lr": 3e-3},
            "data": {"source": "synthetic", "num_documents": docs, "synthetic_doc_len": 96, "synthetic_topics": 4},
            "transport": {"host": "127.0.0.1", "port": 0, "auth_key": "dynamics", "heartbeat_timeout": 30.0},
            "sharded": {"num_shards": 2},
            "run": {"generations": rounds, "batch_size": 4, "local_workers": workers, "seed": seed}}


def _merge(base: dict, over: dict) -> dict:
    out = {k: dict(v) if isinstance(v, dict) else v for k, v in base.items()}
    for k, v in over.items():
        out.setdefault(k, {}).update(v)
    return out


def held_out_documents(cfg: LaunchConfig, n: int = 64) -> list[torch.Tensor]:
    """Documents of the same topics as the training set, from another seed."""
    d = cfg.data
    return synthetic_documents(vocab_size=cfg.model.vocab_size, num_documents=n, doc_len=d.synthetic_doc_len,
                               topics=d.synthetic_topics, seed=cfg.run.seed + 1000)


def best_path_perplexity(model_cfg, bank, docs) -> float:
    """exp of the mean over documents of each document's lowest per-token loss."""
    losses = path_losses(docs, model_cfg, bank, model_cfg.sequence_length)
    return float(math.exp(losses.min(dim=1).values.mean()))


def _bank_from(model_cfg, states) -> dict:
    bank = build_module_bank(model_cfg, seed=0)
    for k, sd in states.items():
        bank[k].load_state_dict(sd)
    return bank


def run_arm(arm: str, base: dict) -> dict:
    if arm not in ARMS:
        raise ValueError(f"unknown arm {arm!r} (one of {sorted(ARMS)})")
    over = ARMS[arm]
    cfg = LaunchConfig.from_dict(_merge(base, over or {}))
    model, diloco = dipaco_config(cfg.model), diloco_config(cfg.diloco)
    t0 = time.monotonic()
    if over is None:
        corpus = build_server_corpus(cfg, model)
        eng = DiPaCoEngine(model, diloco, LocalBackend(model.build_topology()), seed=cfg.run.seed)
        eng.fit(corpus, num_rounds=cfg.run.generations, batch_size=cfg.run.batch_size, log_every=0)
        bank, done = eng.global_modules(), cfg.run.generations
    else:
        server, completed = run_local(cfg)
        done = min(completed.values()) if completed else 0
        if hasattr(server, "merged_bank"):
            bank = _bank_from(model, server.merged_bank())
        else:
            bank = getattr(server, "owner_banks", None)
            if bank is None:  # the coordinator keeps the bank itself
                bank = server.engine.global_modules()
    ppl = best_path_perplexity(model, bank, held_out_documents(cfg))
    return {"arm": arm, "held_out_ppl": round(ppl, 3), "generations": int(done),
            "seconds": round(time.monotonic() - t0, 1)}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--arms", default=",".join(ARMS), help="comma-separated arms")
    ap.add_argument("--rounds", type=int, default=6)
    ap.add_argument("--hidden", type=int, default=64)
    ap.add_argument("--workers", type=int, default=3)
    args = ap.parse_args(argv)
    base = base_config(args.rounds, hidden=args.hidden, workers=args.workers)
    results = [run_arm(a, base) for a in args.arms.split(",") if a]
    anchor = next((r["held_out_ppl"] for r in results if r["arm"] == "sync"), None)
    for r in results:
        if anchor:
            r["vs_sync"] = round(r["held_out_ppl"] / anchor, 3)
        print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
