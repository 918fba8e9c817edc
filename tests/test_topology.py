import pytest

from opendipaco_b200 import DiPaCoConfig, PathTopology, SegmentSpec
from opendipaco_b200.parallel.placement import block_sizes, path_ranks, rank_paths
from opendipaco_b200.topology import is_private_key


def test_paths_and_mixed_radix_roundtrip():
    t = PathTopology((3, 4))
    assert t.num_paths == 12 and len(t.paths()) == 12
    for i, p in enumerate(t.paths()):
        assert t.path_index(p) == i and t.path_from_index(i) == p


def test_module_keys_and_sharing_counts():
    t = PathTopology((4, 4))
    keys = t.module_keys()
    assert keys[0] == "embed" and keys[-1] == "head"
    assert "L0E3" in keys and "L1E0" in keys
    assert t.sharing_count("embed") == 16
    assert t.sharing_count("L0E1") == 4
    assert sorted(t.paths_through_module("L1E2")) == [(e, 2) for e in range(4)]


def test_private_keys_per_path():
    cfg = DiPaCoConfig(level_sizes=[2, 2], embedding="private", head="private")
    t = cfg.build_topology()
    keys = t.module_keys()
    assert "embed" not in keys and "embed.p3" in keys and "head.p0" in keys
    assert all(t.sharing_count(k) == 1 for k in keys if is_private_key(k))
    assert t.path_module_keys((1, 0)) == ["embed.p2", "L0E1", "L1E0", "head.p2"]


def test_advanced_body_segments():
    from opendipaco_b200 import BackboneConfig

    cfg = DiPaCoConfig(backbone=BackboneConfig(layers_per_level=[1]),
                       level_sizes=[1],
                       body=[SegmentSpec(layers=1, sharing="private"), SegmentSpec(layers=2, num_experts=3),
                             SegmentSpec(layers=1)])
    t = cfg.build_topology()
    assert cfg.num_paths == 3 and t.num_paths == 3
    assert t.path_module_keys((2,)) == ["embed", "B1.p2", "L0E2", "B3", "head"]
    assert t.offset_of_key("L0E1") == 1 and t.layers_of_key("L0E1") == 2


def test_sharing_table_lists_paths():
    t = PathTopology((2, 2))
    tab = t.sharing_table()
    assert tab["embed"] == [0, 1, 2, 3] and tab["L0E1"] == [2, 3] and tab["L1E0"] == [0, 2]


def test_config_validation():
    with pytest.raises(ValueError):
        DiPaCoConfig(level_sizes=[2, 2, 2])
    with pytest.raises(ValueError):
        DiPaCoConfig(level_sizes=[0, 2])


def test_placement_balanced_non_divisible():
    assert block_sizes(36, 8) == [5, 5, 5, 5, 4, 4, 4, 4]
    assert block_sizes(16, 8) == [2] * 8
    r = path_ranks(36, 8)
    assert r[:5] == [0] * 5 and r[-4:] == [7] * 4
    assert rank_paths(16, 8, 3) == [6, 7]
    with pytest.raises(ValueError):
        block_sizes(3, 4)
