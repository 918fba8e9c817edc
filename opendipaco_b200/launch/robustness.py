"""Aggregation robustness harness: with a fraction of Byzantine contributors, how far
does the applied update drift from the honest update under the plain weighted mean
(``robustness: off``) versus the coordinate-wise trimmed mean or median (``on``)?
It runs the owners' aggregation primitive directly (``schedule/aggregate.py``), so it
is deterministic and fast.

    python -m opendipaco_b200.launch.robustness --contributors 5 --adversaries 2 --attack signflip

Each round the honest contributors send a shared target direction plus small noise
and the adversaries send an attack: ``signflip`` (the target, negated and boosted),
``largenorm`` (a random direction of large norm) or ``gaussian`` (large noise). The
report is the mean L2 distance of the aggregate from the honest target, relative to
the target's norm. ``trimmed_mean`` drops one value per side per coordinate, so it
tolerates one adversary whatever the contributor count; ``median`` tolerates a
minority (the comparisons of the reference's ``examples/validate_robustness.py``).
"""

from __future__ import annotations

import argparse
import json

import torch

from ..schedule.aggregate import AGGREGATES, robust_delta

ATTACKS = ("signflip", "largenorm", "gaussian")


def _attack(kind: str, target: torch.Tensor, gen: torch.Generator, boost: float) -> torch.Tensor:
    if kind == "signflip":
        return -boost * target
    if kind == "largenorm":
        d = torch.randn(target.shape, generator=gen)
        return d / d.norm() * boost * target.norm()
    if kind == "gaussian":
        return boost * target.norm() / target.numel() ** 0.5 * torch.randn(target.shape, generator=gen)
    raise ValueError(f"attack must be one of {ATTACKS}, got {kind!r}")


def drift(*, contributors: int = 5, adversaries: int = 1, attack: str = "signflip", aggregate: str = "median",
          rounds: int = 50, dim: int = 4096, noise: float = 0.1, boost: float = 10.0, seed: int = 0) -> float:
    """Mean over rounds of ||aggregate - target|| / ||target||."""
    if not 0 <= adversaries <= contributors:
        raise ValueError("adversaries must be between 0 and the contributor count")
    gen = torch.Generator().manual_seed(seed)
    total = 0.0
    for _ in range(rounds):
        target = torch.randn(dim, generator=gen)
        contribs = []
        for i in range(contributors):
            if i < adversaries:
                g = _attack(attack, target, gen, boost)
            else:
                g = target + noise * target.norm() / dim ** 0.5 * torch.randn(dim, generator=gen)
            contribs.append((1.0, [g]))
        delta, wsum = robust_delta(contribs, aggregate=aggregate)
        total += float((delta[0] - target).norm() / target.norm())
    return total / rounds


def table(*, contributors: int = 5, adversaries: int = 1, attack: str = "signflip", **kw) -> dict:
    return {agg: round(drift(contributors=contributors, adversaries=adversaries, attack=attack, aggregate=agg, **kw), 4)
            for agg in AGGREGATES}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--contributors", type=int, default=5)
    ap.add_argument("--adversaries", type=int, default=1)
    ap.add_argument("--attack", choices=ATTACKS, default="signflip")
    ap.add_argument("--rounds", type=int, default=50)
    a = ap.parse_args(argv)
    out = table(contributors=a.contributors, adversaries=a.adversaries, attack=a.attack, rounds=a.rounds)
    print(json.dumps({"contributors": a.contributors, "adversaries": a.adversaries, "attack": a.attack,
                      "relative_drift": out}))


if __name__ == "__main__":
    main()
