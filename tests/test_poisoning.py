"""Poisoning harness (CPU): one worker of four sends boosted sign-flipped
pseudo-gradients; undefended it wrecks the model, the owners' median over a push
quorum keeps it near the clean run.

Behaviour of the reference's ``examples/validate_poisoning.py`` at a small size.
"""

import pytest

from opendipaco_b200.launch.poisoning import run_arm


@pytest.fixture(scope="module")
def results():
    return {a: run_arm(a, rounds=6, boost=50.0) for a in ("clean", "attacked", "robust")}


def test_an_undefended_cluster_is_wrecked(results):
    assert results["attacked"]["held_out_ppl"] > 5 * results["clean"]["held_out_ppl"]


def test_robust_aggregation_holds_the_attack_back(results):
    assert results["robust"]["held_out_ppl"] < 0.5 * results["attacked"]["held_out_ppl"]
    assert results["robust"]["held_out_ppl"] < 4 * results["clean"]["held_out_ppl"]
    assert all(r["generations"] >= 6 for r in results.values())
