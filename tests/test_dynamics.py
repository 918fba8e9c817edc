"""Dynamics harness (CPU): the synchronous anchor and the cluster variants train the
same documents and are scored by held-out best-path perplexity; every variant trains
(perplexity clearly below the uniform vocabulary's) and stays near the anchor.

Behaviour of the reference's ``examples/validate_dynamics.py`` at a small size.
"""

import math

import pytest

from opendipaco_b200.launch.dynamics import ARMS, base_config, run_arm


@pytest.fixture(scope="module")
def anchor():
    return run_arm("sync", base_config(3, docs=96, workers=2))


@pytest.mark.parametrize("arm", ["int4", "delta_down", "decentralized"])
def test_variants_train_near_the_synchronous_anchor(arm, anchor):
    r = run_arm(arm, base_config(3, docs=96, workers=2))
    vocab = 128
    assert r["generations"] >= 3 and math.isfinite(r["held_out_ppl"])
    assert r["held_out_ppl"] < 0.75 * vocab and anchor["held_out_ppl"] < 0.75 * vocab
    assert r["held_out_ppl"] < 2.5 * anchor["held_out_ppl"], (r, anchor)


def test_unknown_arm():
    with pytest.raises(ValueError):
        run_arm("gossip", base_config(1))
    assert "sync" in ARMS and ARMS["sync"] is None
