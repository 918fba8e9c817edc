import json

import pytest
import torch

from opendipaco_b200 import (DiLoCoConfig, DiPaCoConfig, DiPaCoEngine, LocalBackend,
                             latest_checkpoint, load_checkpoint, save_checkpoint)

from helpers import banks_equal, engine, rr_corpus, tiny_config


def test_roundtrip(tmp_path):
    cfg = tiny_config()
    corpus = rr_corpus(cfg)
    a = engine(cfg)
    a.fit(corpus, 3, 8, log_every=0)
    save_checkpoint(a, tmp_path / "c", corpus=corpus, extra={"note": 1})
    meta = json.loads((tmp_path / "c" / "meta.json").read_text())
    assert meta["global_round"] == 3 and meta["world_size"] == 1
    b = engine(cfg, seed=99)
    assert not banks_equal(a.bank, b.bank)
    out = load_checkpoint(b, tmp_path / "c")
    assert banks_equal(a.bank, b.bank) and b._global_round == 3
    assert "corpus" in out and out["extra"] == {"note": 1}


@pytest.mark.parametrize("mat", ["eager", "serial"])
def test_resume_bit_for_bit(tmp_path, mat):
    cfg = tiny_config()
    corpus = rr_corpus(cfg)
    ref = engine(cfg, mat)
    ref.fit(corpus, 6, 8, log_every=0, total_rounds=6)
    a = engine(cfg, mat)
    a.fit(corpus, 3, 8, log_every=0, total_rounds=6)
    save_checkpoint(a, tmp_path / "mid")
    b = engine(cfg, mat, seed=5)
    load_checkpoint(b, tmp_path / "mid")
    b.fit(corpus, 3, 8, log_every=0)
    assert b.total_rounds == 6 and banks_equal(ref.bank, b.bank)


def test_fingerprint_mismatch(tmp_path):
    cfg = tiny_config()
    a = engine(cfg)
    a.fit(rr_corpus(cfg), 1, 8, log_every=0)
    save_checkpoint(a, tmp_path / "c")
    other = DiPaCoConfig(backbone=cfg.backbone, level_sizes=[2, 2], sequence_length=32)
    bad = DiPaCoEngine(other, DiLoCoConfig(inner_steps=4), LocalBackend(other.build_topology()))
    with pytest.raises(ValueError, match="fingerprint"):
        load_checkpoint(bad, tmp_path / "c")
    load_checkpoint(bad, tmp_path / "c", strict=False)


def test_latest_checkpoint(tmp_path):
    cfg = tiny_config()
    a = engine(cfg)
    corpus = rr_corpus(cfg)
    for r in range(3):
        a.fit(corpus, 1, 8, log_every=0)
        save_checkpoint(a, tmp_path / f"r{r}")
    assert latest_checkpoint(tmp_path).endswith("r2")
    assert latest_checkpoint(tmp_path / "nope") is None


def test_checkpoint_loads_in_reference(tmp_path, reference_pkg):
    """Our rank file is readable by the reference engine (same schema + fingerprint)."""
    R = reference_pkg
    cfg = tiny_config()
    a = engine(cfg)
    a.fit(rr_corpus(cfg), 2, 8, log_every=0)
    state = a.state_dict()
    rcfg = R.DiPaCoConfig(backbone=R.BackboneConfig(**vars(cfg.backbone)), level_sizes=[2, 2],
                          sequence_length=16)
    r = R.DiPaCoEngine(rcfg, R.DiLoCoConfig(inner_steps=4, inner_lr=1e-3),
                       R.LocalBackend(rcfg.build_topology()), seed=7)
    r.load_state_dict(state)
    for k in a.bank:
        for x, y in zip(a.bank[k].state_dict().values(), r.bank[k].state_dict().values()):
            assert torch.equal(x, y)
