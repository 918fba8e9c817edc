"""Owner churn on a live sharded cluster (CPU, loopback TCP): tracker, signed-epoch
scheduler, four dynamic owners and two reconnecting workers train a few generations
while one owner crashes, leaves, flaps, sleeps past the grace, or a fifth joins.

Mirrors the arms of the reference's ``examples/validate_churn.py`` (``run_arm``): every
arm must finish its generations; a departure is failed over (the leaving owner is out
of the epoch and every key is served by live owners), a flap shorter than the grace is
absorbed without a new epoch, a sleeper is removed and re-added to the same placement,
and a joiner is folded in with its keys synced before it serves them.
"""

import pytest

from opendipaco_b200.launch.churn import ARMS, ChurnCluster, run_arm


@pytest.mark.parametrize("arm", ARMS)
def test_churn_arm(arm):
    m = run_arm(arm, rounds=2)
    assert m["survived"], m
    if arm in ("none", "flap"):
        assert m["epochs"] == 0 and m["remaps"] == 0, m
    elif arm in ("abrupt", "graceful"):
        assert m["epochs"] >= 1 and m["remaps"] >= 1 and m["failover_s"] is not None, m
    elif arm == "suspend":
        # removed (one epoch), re-added (another): rendezvous hashing restores the placement
        assert m["epochs"] >= 2 and m["remaps"] == 0 and m["settle_s"] is not None, m
    elif arm == "join":
        assert m["epochs"] >= 1 and m["remaps"] >= 1 and m["settle_s"] is not None, m


def test_graceful_leave_fails_over_without_waiting_out_the_grace():
    """The leaver tombstones itself, so the next epoch comes at the rate limit, not after
    the tracker TTL plus the owner grace."""
    m = run_arm("graceful", rounds=2, owner_grace=5.0)
    assert m["survived"] and m["failover_s"] is not None and m["failover_s"] < 5.0, m


def test_unknown_arm_is_rejected():
    with pytest.raises(ValueError):
        run_arm("meteor")
    assert ChurnCluster().k == 3
