"""Aggregation robustness harness (launch/robustness.py): with Byzantine contributors
the plain mean drifts far from the honest update; the trimmed mean holds against one
adversary but not two; the median holds against a minority; with no adversary all
three stay close. Behaviour of the reference's ``examples/validate_robustness.py``."""

import pytest

from opendipaco_b200.launch.robustness import ATTACKS, drift, table


@pytest.mark.parametrize("attack", ATTACKS)
def test_one_adversary_of_five(attack):
    t = table(contributors=5, adversaries=1, attack=attack, rounds=10, dim=512)
    assert t["trimmed_mean"] < 0.2 and t["median"] < 0.2
    assert t["mean"] > 2 * t["median"]


def test_breakdown_points():
    two = table(contributors=5, adversaries=2, attack="signflip", rounds=10, dim=512)
    assert two["trimmed_mean"] > 1.0 > 0.3 > two["median"]
    clean = table(contributors=5, adversaries=0, rounds=10, dim=512)
    assert max(clean.values()) < 0.1
    with pytest.raises(ValueError):
        drift(contributors=3, adversaries=4)
