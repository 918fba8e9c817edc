"""Poisoning harness: one worker of a sharded cluster sends boosted, sign-flipped
pseudo-gradients; how much does each owner-side defense hold it back? Every arm trains
the same documents for the same generations and is scored by held-out best-path
perplexity (as in ``launch/dynamics.py``).

    python -m opendipaco_b200.launch.poisoning --rounds 6

Arms (the comparisons of the reference's ``examples/validate_poisoning.py``):

* ``clean``     -- honest workers only, no defense (the reference point);
* ``attacked``  -- one of the workers multiplies its pseudo-gradients by ``-boost``;
* ``clipped``   -- the same attack, owners clip every pushed pseudo-gradient to
  ``max_update_norm``;
* ``robust``    -- the same attack, owners buffer pushes to a quorum and apply the
  coordinate-wise median (plus the clip).
"""

from __future__ import annotations

import argparse
import dataclasses
import json
import threading
import time

from ..schedule import ParameterServer, Scheduler, run_sharded_worker
from .config import LaunchConfig, diloco_config, dipaco_config
from .dynamics import base_config, best_path_perplexity, held_out_documents
from .roles import build_server_corpus

ARMS = ("clean", "attacked", "clipped", "robust")


def _poison(boost: float):
    def hook(path, contrib):
        scaled = {k: [-boost * g for g in gs] for k, gs in contrib.shared_delta.items()}
        return dataclasses.replace(contrib, shared_delta=scaled)
    return hook


def run_arm(arm: str, *, rounds: int = 6, honest: int = 3, boost: float = 20.0, clip: float = 10.0,
            seed: int = 0) -> dict:
    if arm not in ARMS:
        raise ValueError(f"unknown arm {arm!r} (one of {ARMS})")
    cfg = LaunchConfig.from_dict(base_config(rounds, workers=honest, seed=seed))
    model, diloco = dipaco_config(cfg.model), diloco_config(cfg.diloco)
    corpus = build_server_corpus(cfg, model)
    keys = model.build_topology().module_keys()
    defense = {}
    if arm in ("clipped", "robust"):
        defense["max_update_norm"] = clip
    if arm == "robust":
        defense.update(robustness="on", aggregate="median", quorum_target=3, quorum_timeout=1.0)
    ps = ParameterServer(model, keys, diloco, host="127.0.0.1", auth_key="poison", **defense)
    ps.start()
    sched = Scheduler(model, corpus, [("127.0.0.1", ps.port)], diloco, cfg.run.batch_size, host="127.0.0.1",
                      auth_key="poison", seed=seed)
    sched.start()
    stop = threading.Event()
    hooks = [None] * honest + ([_poison(boost)] if arm != "clean" else [])
    ws = [threading.Thread(target=run_sharded_worker, args=(model, diloco, ("127.0.0.1", sched.port)),
                           kwargs=dict(seed=i, auth_key="poison", stop_event=stop, heartbeat_interval=1.0,
                                       contribution_hook=h), daemon=True) for i, h in enumerate(hooks)]
    t0 = time.monotonic()
    for w in ws:
        w.start()
    try:
        done = sched.fit(num_generations=rounds)
        with ps._lock:
            for k in list(ps._buffers):
                ps._flush_buffer(k)
        ppl = best_path_perplexity(model, ps.bank, held_out_documents(cfg))
    finally:
        stop.set()
        sched.shutdown()
        ps.shutdown()
        for w in ws:
            w.join(timeout=15)
    return {"arm": arm, "held_out_ppl": round(ppl, 3), "generations": int(min(done.values())),
            "norm_clipped": ps.metrics.summary()["norm_clipped"], "seconds": round(time.monotonic() - t0, 1)}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--arms", default=",".join(ARMS))
    ap.add_argument("--rounds", type=int, default=6)
    ap.add_argument("--boost", type=float, default=20.0)
    args = ap.parse_args(argv)
    for a in args.arms.split(","):
        print(json.dumps(run_arm(a, rounds=args.rounds, boost=args.boost)), flush=True)


if __name__ == "__main__":
    main()
