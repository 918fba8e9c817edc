import math

import pytest
import torch

from opendipaco_b200.schedule import compress as C


def test_int8_error_feedback_is_exact_in_sum():
    torch.manual_seed(0)
    d = [torch.randn(64, 32), torch.randn(10)]
    payload, resid = C.compress_delta(d, "int8")
    rec = C.maybe_dequantize(payload)
    for a, b, r in zip(d, rec, resid):
        assert torch.allclose(a, b + r, atol=1e-6)


def test_int4_group_payload_layout():
    x = torch.tensor([0.7, -0.7, 0.1, 0.0] + [0.0] * 124)
    p, r = C._quantize_int4(x)
    assert p["g"] == 128 and p["n"] == 128 and p["q4"].numel() == 64
    # 0.7 -> +7 (+8 -> 15), -0.7 -> -7 (+8 -> 1): high nibble first
    assert int(p["q4"][0]) == (15 << 4) | 1
    assert torch.allclose(C._dequant_int4(p)[:2], torch.tensor([0.7, -0.7]), atol=1e-6)


def test_sparse_topk_rows_and_residual():
    torch.manual_seed(1)
    d = torch.randn(8, 100)
    p, r = C.compress_delta([d], "none", density=0.1)
    assert p[0]["i"].numel() == 8 * 10
    dense = C.maybe_dequantize(p)[0]
    assert torch.allclose(dense + r[0], d)
    assert (dense != 0).sum(1).eq(10).all()


def test_state_delta_roundtrip_and_validation():
    torch.manual_seed(2)
    base = {"w": torch.randn(16, 16), "step": torch.tensor(3)}
    cur = {"w": base["w"] + 0.01 * torch.randn(16, 16), "step": torch.tensor(4)}
    for mode in ("int8", "int4"):
        enc = C.encode_state_delta(cur, base, mode)
        out = C.apply_state_delta(base, enc)
        assert torch.allclose(out["w"], cur["w"], atol=5e-3) and out["step"] == 4
    with pytest.raises(ValueError):
        C.maybe_dequantize([{"sp": [4], "i": torch.tensor([9], dtype=torch.int32), "v": torch.ones(1)}])
    with pytest.raises(ValueError):
        C._dequant_int4({"q4": torch.zeros(3, dtype=torch.uint8), "s": torch.ones(1), "g": 128, "n": 128})
    with pytest.raises(TypeError):
        C.maybe_dequantize(["nope"])


def test_digests_stable_under_noise_and_sensitive_to_change():
    torch.manual_seed(3)
    g = {"L0E0": [torch.randn(50, 50)]}
    noisy = {"L0E0": [g["L0E0"][0] + 1e-9]}
    assert C.pseudograd_digest(g) == C.pseudograd_digest(noisy)
    assert C.pseudograd_digest(g) != C.pseudograd_digest({"L0E0": [g["L0E0"][0] * 2]})
    assert C.state_digest({"w": torch.ones(3)}) == C.state_digest({"w": torch.ones(3)})


def test_wire_roundtrip_and_reference_compat(reference_pkg):
    from opendipaco.schedule import wire as RW

    from opendipaco_b200.schedule import wire as W

    msg = {"type": "task", "path": (1, 2), "w": torch.randn(3, 4).to(torch.bfloat16),
           "ids": torch.arange(5, dtype=torch.int32), "x": None, "f": 1.5, "l": [True, "s"]}
    raw = W.encode(msg)
    assert raw == RW.encode(msg)
    back = W.decode(raw)
    assert back["path"] == (1, 2) and torch.equal(back["w"], msg["w"]) and back["l"] == [True, "s"]
    with pytest.raises(TypeError):
        W.encode({1: 2})
    assert math.isfinite(back["f"])


def test_payloads_and_digests_match_reference(reference_pkg):
    """Uploads encoded here decode to the same values in the reference and vice versa,
    the payload bytes on the wire are identical, and audit digests agree."""
    from opendipaco.schedule import compress as RC
    from opendipaco.schedule import wire as RW

    torch.manual_seed(7)
    delta = [torch.randn(12, 40), torch.randn(333), torch.zeros(5)]
    for mode, density in (("int8", 1.0), ("int4", 1.0), ("bf16", 1.0), ("int8", 0.1), ("int4", 0.05),
                          ("none", 0.2)):
        ours, ours_r = C.compress_delta(delta, mode, density=density)
        theirs, theirs_r = RC.compress_delta(delta, mode, density=density)
        assert RW.encode({"p": ours}) == RW.encode({"p": theirs}), (mode, density)
        for a, b in zip(C.maybe_dequantize(theirs), RC.maybe_dequantize(ours)):
            assert torch.equal(a, b)
        for a, b in zip(ours_r, theirs_r):
            assert torch.equal(a, b)
    g = {"L0E0": delta, "embed": [torch.randn(7, 3)]}
    assert C.pseudograd_digest(g) == RC.pseudograd_digest(g)
    sd = {"w": torch.randn(4, 4), "n": torch.arange(3)}
    assert C.state_digest(sd) == RC.state_digest(sd)
    base = {"w": torch.randn(6, 6)}
    cur = {"w": base["w"] + 0.1}
    for mode in ("int8", "int4"):
        enc = C.encode_state_delta(cur, base, mode)
        assert RW.encode(enc) == RW.encode(RC.encode_state_delta(cur, base, mode))
        assert torch.equal(RC.apply_state_delta(base, enc)["w"], C.apply_state_delta(base, enc)["w"])
