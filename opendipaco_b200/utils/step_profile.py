"""Where an inner step's device time goes: every extension call of the fused executor's
inner step is bracketed by CUDA events (warm caches, steady state, no profiler), and the
times are summed per kernel and epilogue.

    python -m opendipaco_b200.utils.step_profile [--levels 4 4] [--batch 24] [--steps 3] [--graph]

Defaults: the 16-path 4x4 DiPaCo, hidden 384, 6 heads, ffn 1024, layers [2, 2], vocab
32000, 24 sequences of 128 tokens per path, 20 inner steps a round. The CPU is put ahead
of the GPU (a sleep kernel first) so that an event pair measures its kernel, not launch
latency. ``other`` is the step's total minus the listed calls (torch fills and copies).
"""

from __future__ import annotations

import argparse
import collections
import json

import torch

from ..ops import _ext


class _Recorder:
    """Stands in for the extension module: calls pass through, each bracketed by events."""

    def __init__(self, mod, stream):
        self._mod, self._st, self.events = mod, stream, []

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if not callable(fn):
            return fn

        def call(*a, **kw):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(self._st)
            out = fn(*a, **kw)
            e1.record(self._st)
            tag = name
            if name == "gemm_bf16":
                # (A, lda, sa, amn, B, ldb, sb, bmn, C, ldc, sc, M, N, K, G, epi, ...)
                tag = f"gemm M{a[11]} N{a[12]} K{a[13]} epi{a[15]} A{'mn' if a[3] else 'k'} B{'mn' if a[7] else 'k'}"
            self.events.append((tag, e0, e1))
            return out

        return call


def profile_inner_step(ex, steps: int = 3) -> dict:
    """Per-call device times of ``steps`` eager inner steps of fused executor ``ex``
    (its round inputs must already be staged, e.g. by one ``engine.fit`` round)."""
    st = torch.cuda.current_stream()
    real = _ext.ext()
    rec = _Recorder(real, st)
    totals = collections.defaultdict(lambda: [0, 0.0])
    step_ms = 0.0
    _ext._mod = rec
    try:
        for s in range(steps):
            torch.cuda.synchronize()
            torch.cuda._sleep(200_000_000)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(st)
            ex._step(s % ex.IDS.shape[0])
            b.record(st)
            torch.cuda.synchronize()
            step_ms += a.elapsed_time(b)
            for tag, e0, e1 in rec.events:
                totals[tag][0] += 1
                totals[tag][1] += e0.elapsed_time(e1)
            rec.events.clear()
    finally:
        _ext._mod = real
    rows = sorted(((t, n // steps, ms / steps) for t, (n, ms) in totals.items()), key=lambda r: -r[2])
    listed = sum(r[2] for r in rows)
    step = step_ms / steps
    return {"step_ms": step, "calls": [{"call": t, "per_step": n, "ms": round(ms, 4),
                                        "share": round(ms / step, 4)} for t, n, ms in rows],
            "other_ms": round(step - listed, 4)}


def graph_step_ms(ex, rounds: int = 5) -> float:
    """Device time of one inner step inside the captured round graph (a round's replay
    divided by its inner steps; median of ``rounds`` replays after one warm-up)."""
    steps = ex.e.diloco.inner_steps
    ex._run_inner(steps)
    torch.cuda.synchronize()
    times = []
    for _ in range(rounds):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        ex._run_inner(steps)
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    times.sort()
    return times[len(times) // 2] / steps


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--levels", type=int, nargs=2, default=[4, 4])
    ap.add_argument("--batch", type=int, default=24)
    ap.add_argument("--seq", type=int, default=128)
    ap.add_argument("--hidden", type=int, default=384)
    ap.add_argument("--heads", type=int, default=6)
    ap.add_argument("--ffn", type=int, default=1024)
    ap.add_argument("--vocab", type=int, default=32000)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--graph", action="store_true",
                    help="also time whole rounds replayed from the CUDA graph (no per-call events)")
    args = ap.parse_args()

    from .. import BackboneConfig, DiLoCoConfig, DiPaCoConfig, DiPaCoEngine, LocalBackend
    from ..data import ShardedCorpus, zipf_documents

    bb = BackboneConfig(vocab_size=args.vocab, hidden_size=args.hidden, num_attention_heads=args.heads,
                        intermediate_size=args.ffn, layers_per_level=[2, 2], max_position_embeddings=2048)
    cfg = DiPaCoConfig(backbone=bb, level_sizes=list(args.levels), sequence_length=args.seq)
    dl = DiLoCoConfig(inner_steps=20, inner_autocast=True)
    P = cfg.num_paths
    docs = zipf_documents(vocab_size=args.vocab, num_documents=200 * P, min_len=args.seq, max_len=4 * args.seq,
                          seed=0)
    corpus = ShardedCorpus.from_assignments(docs, torch.arange(len(docs)) % P, P, args.seq)
    eng = DiPaCoEngine(cfg, dl, LocalBackend(cfg.build_topology()), device=torch.device("cuda"), seed=0)
    eng.fit(corpus, num_rounds=1, batch_size=args.batch, log_every=0)
    if args.graph:
        print(json.dumps({"graph_step_ms": round(graph_step_ms(eng._fused), 4)}))
    out = profile_inner_step(eng._fused, args.steps)
    print(json.dumps({"config": vars(args), "step_ms": round(out["step_ms"], 4), "other_ms": out["other_ms"]}))
    for row in out["calls"]:
        print(json.dumps(row))


if __name__ == "__main__":
    main()
