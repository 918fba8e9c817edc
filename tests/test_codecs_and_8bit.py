"""Wire codecs under hostile input and the 8-bit inner optimizer (CPU).

Codecs: int4 groups adapt their scale, int4 / sparse / delta payloads decode within
their bounds, sparse error feedback eventually sends every dropped entry, density 1 is
the dense payload, malformed payloads are refused, and a payload declaring a huge shape
is refused by the coordinator and the owners before anything is allocated.
8-bit Adam: blockwise moments within their quantization bound, the update tracks fp32
AdamW, the state is small and round-trips through ``state_dict``, the factory selects
it, and it trains a path. Activation checkpointing in the module executor is bit-exact.

Behaviours of the reference's ``tests/test_w2_int4.py``, ``tests/test_w2_sparse.py``,
``tests/test_w3_quant.py`` and ``tests/test_w3_checkpoint.py``.
"""

import pytest
import torch

from opendipaco_b200 import DiLoCoConfig
from opendipaco_b200.optim.adam8bit import Adam8bit, dequantize_m, dequantize_v, quantize_m, quantize_v
from opendipaco_b200.optim.diloco import make_inner_optimizer
from opendipaco_b200.schedule import AsyncScheduler, CoordinatorServer, ParameterServer, PeerIdentity, make_grant
from opendipaco_b200.schedule import compress as C

from helpers import engine, rr_corpus, tiny_config


# ------------------------------------------------------------------ int4 and sparse
def test_int4_scale_adapts_per_group_and_round_trips():
    x = torch.cat([torch.full((128,), 1e-3), torch.full((128,), 10.0)])
    x[::7] *= -1
    p, resid = C._quantize_int4(x)
    rec = C._dequant_int4(p)
    assert (rec[:128] - x[:128]).abs().max() <= 1e-3 / 7 + 1e-9      # the small group keeps its own scale
    assert (rec[128:] - x[128:]).abs().max() <= 10.0 / 7 + 1e-6
    torch.testing.assert_close(rec + resid, x)
    shaped = C._Int4.decode_shaped(C._Int4.encode(torch.randn(3, 50))[0])
    assert shaped.shape == (3, 50)


@pytest.mark.parametrize("mode", ["int8", "int4", "none"])
def test_sparse_error_feedback_eventually_sends_the_dropped_mass(mode):
    torch.manual_seed(0)
    d = torch.randn(6, 40)
    carry, sent = None, torch.zeros_like(d)
    for r in range(20):  # one delta, then nothing new: 10% density drains the carried residual
        payload, resid = C.compress_delta([d if r == 0 else torch.zeros_like(d)], mode, carry=carry, density=0.1)
        sent += C.maybe_dequantize(payload)[0]
        carry = resid
    torch.testing.assert_close(sent + carry[0], d, rtol=0, atol=1e-5)  # mass is conserved
    if mode == "none":  # ten rounds of 10% send every entry exactly
        assert (sent != 0).all() and carry[0].abs().max() == 0
    else:               # quantization leaves a residual that keeps draining
        assert carry[0].abs().max() < 0.25 * d.abs().max() and (sent != 0).float().mean() > 0.9


def test_density_one_is_the_dense_payload():
    d = [torch.randn(4, 9), torch.randn(7)]
    dense, _ = C.compress_delta(d, "int8")
    full, _ = C.compress_delta(d, "int8", density=1.0)
    for a, b in zip(dense, full):
        assert torch.equal(a["q"], b["q"]) and a["s"] == b["s"]


@pytest.mark.parametrize("payload", [
    {"q4": torch.zeros(3, dtype=torch.uint8), "s": torch.ones(1), "g": 128, "n": 128},      # too few codes
    {"q4": torch.zeros(64, dtype=torch.uint8), "s": torch.ones(2), "g": 128, "n": 128},     # too many scales
    {"q4": torch.zeros(64, dtype=torch.uint8), "s": torch.ones(1), "g": "x", "n": 128},
    {"sp": [4, 4], "i": torch.tensor([0, 99], dtype=torch.int32), "v": torch.ones(2)},      # index out of range
    {"sp": [4, -4], "i": torch.tensor([0], dtype=torch.int32), "v": torch.ones(1)},
    {"sp": [4, 4], "i": torch.tensor([0, 1], dtype=torch.int32), "v": torch.ones(3)},       # length mismatch
])
def test_malformed_payloads_are_refused(payload):
    with pytest.raises((ValueError, TypeError, KeyError)):
        C.maybe_dequantize([payload])


def _huge_sparse():
    return {"sp": [1 << 20, 1 << 20], "i": torch.tensor([0], dtype=torch.int32), "v": torch.ones(1)}


def test_huge_declared_shapes_are_refused_before_allocation():
    with pytest.raises(ValueError):
        C.decode_checked([_huge_sparse()], [(4, 4)])
    cfg = tiny_config()
    # the owner
    sched = PeerIdentity.generate()
    keys = cfg.build_topology().module_keys()
    ps = ParameterServer(cfg, keys, DiLoCoConfig(inner_steps=2), host="127.0.0.1", scheduler_pub=sched.public_key_hex)
    try:
        key = keys[0]
        grad = [_huge_sparse() for _ in ps.bank[key].parameters()]
        ack = ps._push({"grant": make_grant((0, 0), [key], 1.0, "t", identity=sched), "updates": {key: {"grad": grad}},
                        "private": {}})
        assert not ack["applied"] and ps.metrics.summary()["invalid_rejected"] == 1
    finally:
        ps.shutdown()
    # the coordinator, with a wrong private state too
    e = engine(cfg)
    coord = CoordinatorServer(AsyncScheduler(e), rr_corpus(cfg), 2, host="127.0.0.1")
    key = next(k for k in coord._versions)
    n_params = len(list(e.bank[key].parameters()))
    shared, _, valid = coord._decode_upload({"shared_grad": {key: [_huge_sparse()] * n_params},
                                             "loss": 1.0})
    assert not valid
    pcfg = tiny_config(embedding="private")
    pe = engine(pcfg)
    pc = CoordinatorServer(AsyncScheduler(pe), rr_corpus(pcfg), 2, host="127.0.0.1")
    bad = {"embed.p0": {"embed_tokens.weight": torch.zeros(3, 3)}}
    assert not pc._decode_upload({"shared_grad": {}, "private_weights": bad, "loss": 1.0})[2]


# ------------------------------------------------------------------ 8-bit Adam
def test_blockwise_moments_round_trip_within_their_bound():
    torch.manual_seed(0)
    m = torch.randn(1000) * torch.logspace(-4, 0, 1000)
    q, absmax = quantize_m(m)
    rec = dequantize_m(q, absmax).reshape(-1)[:1000]
    per_block = absmax.repeat_interleave(q.shape[1])[:1000]
    assert ((rec - m).abs() <= per_block / 127 * 0.5 + 1e-12).all()
    v = torch.rand(1000) * 1e-3
    qv, lo, scale = quantize_v(v)
    recv = dequantize_v(qv, lo, scale).reshape(-1)[:1000]
    assert (recv >= 0).all() and (recv - v).abs().max() <= scale.max() * 0.5 + 1e-12


def test_adam8bit_tracks_fp32_adamw_and_its_state_is_small():
    torch.manual_seed(0)
    w0 = torch.randn(64, 128)
    a, b = torch.nn.Parameter(w0.clone()), torch.nn.Parameter(w0.clone())
    oa = torch.optim.AdamW([a], lr=1e-3, weight_decay=0.01)
    ob = Adam8bit([b], lr=1e-3, weight_decay=0.01)
    for step in range(20):
        g = torch.randn(64, 128)
        a.grad, b.grad = g.clone(), g.clone()
        oa.step()
        ob.step()
    moved = (a.detach() - w0).abs().mean()
    assert (a.detach() - b.detach()).abs().mean() < 0.05 * moved
    st = ob.state[b]
    nbytes = sum(t.numel() * t.element_size() for t in st.values() if torch.is_tensor(t))
    assert nbytes < 0.3 * 8 * b.numel()  # vs two fp32 moments
    other = Adam8bit([torch.nn.Parameter(w0.clone())], lr=1e-3, weight_decay=0.01)
    other.load_state_dict(ob.state_dict())
    st2 = next(iter(other.state.values()))
    assert st2["m_q"].dtype == torch.int8 and st2["v_q"].dtype == torch.uint8
    assert torch.equal(st2["m_q"], st["m_q"]) and st2["step"] == st["step"]


def test_factory_selects_8bit_and_it_trains_a_path():
    lin = torch.nn.Linear(4, 4)
    assert isinstance(make_inner_optimizer(lin, DiLoCoConfig(optim_8bit=True)), Adam8bit)
    assert isinstance(make_inner_optimizer(lin, DiLoCoConfig()), torch.optim.AdamW)
    cfg = tiny_config()
    e = engine(cfg, inner_steps=4, inner_lr=3e-2, optim_8bit=True)
    hist = e.fit(rr_corpus(cfg), num_rounds=3, batch_size=2, log_every=0)
    assert hist[-1].inner_loss < hist[0].inner_loss


# ------------------------------------------------------------------ activation checkpointing
def test_activation_checkpointing_is_bit_exact():
    cfg = tiny_config(layers=[2, 2])
    plain = engine(cfg, inner_steps=3, inner_lr=1e-2)
    ckpt = engine(cfg, inner_steps=3, inner_lr=1e-2, activation_checkpoint=True)
    corpus = rr_corpus(cfg)
    plain.fit(corpus, num_rounds=2, batch_size=2, log_every=0)
    ckpt.fit(corpus, num_rounds=2, batch_size=2, log_every=0)
    for k in plain.bank:
        for x, y in zip(plain.bank[k].parameters(), ckpt.bank[k].parameters()):
            assert torch.equal(x, y), k
