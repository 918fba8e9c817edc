"""Budget calculators (utils/budget.py): per-parameter wire bytes of each payload
format, sync traffic scaling as 1 / inner_steps, and the memory table's levers.
Behaviour of the reference's ``examples/bandwidth_budget.py`` / ``vram_budget.py``."""

import pytest

from opendipaco_b200.utils.budget import bandwidth_table, main, per_param_bytes, vram_table


def test_per_param_bytes_follow_the_payload_formats():
    assert per_param_bytes("none") == (4.0, 4.0)
    assert per_param_bytes("bf16") == (2.0, 2.0)
    assert per_param_bytes("int8") == (2.0, 1.0)                     # weights stay bf16 without a keyframe
    assert per_param_bytes("int8", "delta") == (1.0, 1.0)
    d, u = per_param_bytes("int4", "delta")
    assert d == u == pytest.approx(0.5 + 4 / 128)                     # nibbles + one fp32 scale per group
    assert per_param_bytes("int8", "delta", 0.1)[1] == pytest.approx(0.1 * (4 + 1))
    with pytest.raises(ValueError):
        per_param_bytes("fp8")
    with pytest.raises(ValueError):
        per_param_bytes("int8", density=0.0)


def test_sync_traffic_scales_inversely_with_inner_steps():
    rows = bandwidth_table(params=1e8, tokens=1e9, batch=8, seq_len=1024, inner_steps=(50, 100),
                           modes=[("int8", "delta", 1.0)])
    assert rows[0]["up_GB"] == pytest.approx(2 * rows[1]["up_GB"], rel=1e-3)
    assert rows[0]["uplink_hours"] > rows[1]["uplink_hours"] > 0


def test_memory_table_and_cli(capsys):
    t = vram_table(hidden=64, heads=4, kv_heads=None, ffn=128, layers=[1, 1], vocab=256, levels=[2, 2], batch=4,
                   seq_len=64, paths_per_gpu=2)
    assert t["module_executor_bf16_ckpt"]["total"] < t["module_executor"]["total"]
    assert t["fused_executor"]["total"] > 0
    main(["bandwidth", "--params", "1e6", "--tokens", "1e8"])
    assert capsys.readouterr().out.count("\n") == 20
