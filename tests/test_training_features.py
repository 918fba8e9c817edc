"""Training-side features on CPU: the inner LR schedule across rounds and fit calls,
validation tracking with the best state per path, bf16 autocast keeping fp32 masters,
EM helpers (top-k routing, overlapping shards, loss-based re-sharding), the memory
estimator and the worker's shard cache.

Behaviours of the reference's ``tests/test_warmstart_schedule.py``,
``tests/test_early_stopping.py``, ``tests/test_heterogeneity.py`` (autocast),
``tests/test_em_overlap.py``, ``tests/test_w3_memory.py`` and ``tests/test_shard_cache.py``.
"""

import math

import pytest
import torch

from opendipaco_b200 import DiLoCoConfig
from opendipaco_b200.data import ShardedCorpus
from opendipaco_b200.em import assign_paths_by_loss, path_losses, reshard_by_loss
from opendipaco_b200.optim.diloco import inner_lr_at, make_inner_optimizer
from opendipaco_b200.routing import KMeansRouter
from opendipaco_b200.schedule.distributed import ShardCache
from opendipaco_b200.train.memory import _count_params, fits, vram_breakdown

from helpers import banded_docs, engine, rr_corpus, tiny_config


# ------------------------------------------------------------------ inner LR schedule
def test_constant_and_cosine_schedules():
    const = DiLoCoConfig(inner_lr=1e-3, inner_lr_schedule="constant")
    assert {inner_lr_at(s, 100, const) for s in range(100)} == {1e-3}
    cos = DiLoCoConfig(inner_lr=1e-3, inner_min_lr_ratio=0.1)
    assert inner_lr_at(50, None, cos) == 1e-3  # no horizon: flat
    lrs = [inner_lr_at(s, 100, cos) for s in range(101)]
    assert lrs[0] == pytest.approx(1e-3) and lrs[100] == pytest.approx(1e-4)
    assert all(a >= b for a, b in zip(lrs, lrs[1:]))
    assert lrs[50] == pytest.approx(1e-4 + 0.9e-3 * 0.5)


def test_warmup_then_decay():
    cfg = DiLoCoConfig(inner_lr=2e-3, inner_warmup_steps=4, inner_min_lr_ratio=0.0)
    assert [inner_lr_at(s, 20, cfg) for s in range(4)] == pytest.approx([5e-4, 1e-3, 1.5e-3, 2e-3])
    assert inner_lr_at(4, 20, cfg) == pytest.approx(2e-3) and inner_lr_at(20, 20, cfg) == pytest.approx(0.0)


def test_schedule_is_continuous_across_fit_calls():
    """Two fit() calls of 2 rounds each train exactly like one call of 4: the horizon
    is set once and the step counter carries over."""
    cfg = tiny_config()
    one, two = engine(cfg, inner_steps=3, inner_lr=1e-2), engine(cfg, inner_steps=3, inner_lr=1e-2)
    corpus = rr_corpus(cfg)
    one.fit(corpus, num_rounds=4, batch_size=2, log_every=0)
    two.fit(corpus, num_rounds=2, batch_size=2, log_every=0, total_rounds=4)
    two.fit(corpus, num_rounds=2, batch_size=2, log_every=0)
    assert two.total_rounds == 4
    for k in one.bank:
        for a, b in zip(one.bank[k].parameters(), two.bank[k].parameters()):
            assert torch.equal(a, b), k


def test_schedule_drives_the_optimizer():
    cfg = DiLoCoConfig(inner_lr=1e-3, inner_min_lr_ratio=0.5)
    model = torch.nn.Linear(4, 4)
    opt = make_inner_optimizer(model, cfg)
    assert opt.param_groups[0]["lr"] == pytest.approx(1e-3)
    assert isinstance(opt, torch.optim.AdamW)


# ------------------------------------------------------------------ validation and best state
def test_validation_split_is_deterministic_and_disjoint():
    cfg = tiny_config()
    docs = banded_docs(cfg.backbone.vocab_size, per=12)
    a, b = rr_corpus(cfg, docs, val_fraction=0.25), rr_corpus(cfg, docs, val_fraction=0.25)
    assert a.has_validation
    for p in range(cfg.num_paths):
        assert torch.equal(a.val_shard(p), b.val_shard(p)) and a.val_shard(p).size(0) >= 1
        rows = {tuple(r.tolist()) for r in a.shard(p)}
        assert not rows & {tuple(r.tolist()) for r in a.val_shard(p)} or a.shard(p).size(0) == 0


def test_engine_tracks_the_best_state_and_compose_best_reproduces_it():
    cfg = tiny_config()
    e = engine(cfg, inner_steps=4, inner_lr=3e-2)
    corpus = rr_corpus(cfg, banded_docs(cfg.backbone.vocab_size, per=12), val_fraction=0.25)
    hist = e.fit(corpus, num_rounds=3, batch_size=2, log_every=0)
    assert all(m.val_loss is not None and math.isfinite(m.val_loss) for m in hist)
    for path in e.topology.paths():
        best = e.best_val_loss[path]
        assert best <= min(e.best_val_loss.values()) + 10  # recorded
        model = e.compose_best(path)
        val = corpus.val_shard(e.topology.path_index(path))
        assert e._val_loss(model, val, 2) == pytest.approx(best, rel=1e-5)


# ------------------------------------------------------------------ autocast
def test_inner_autocast_keeps_fp32_masters_and_trains():
    cfg = tiny_config()
    e = engine(cfg, inner_steps=4, inner_lr=3e-2, inner_autocast=True)
    corpus = rr_corpus(cfg)
    hist = e.fit(corpus, num_rounds=3, batch_size=2, log_every=0)
    assert all(p.dtype == torch.float32 for m in e.bank.values() for p in m.parameters())
    assert hist[-1].inner_loss < hist[0].inner_loss


# ------------------------------------------------------------------ EM helpers
def test_kmeans_topk_is_nearest_first():
    cents = torch.tensor([[0.0, 0.0], [10.0, 0.0], [0.0, 5.0]])
    r = KMeansRouter(3)
    r.centroids = cents
    x = torch.tensor([[1.0, 0.0], [9.0, 1.0]])
    assert r.predict_topk(x, 3).tolist() == [[0, 2, 1], [1, 0, 2]]  # squared distances 82 < 97
    assert torch.equal(r.predict_topk(x, 1)[:, 0], r.predict(x))


def test_overlapping_shards_duplicate_documents_and_weight_by_tokens():
    docs = [torch.arange(10) + 100 * i for i in range(4)]
    assign = torch.tensor([[0, 1], [1, 0], [0, 1], [0, 1]])
    c = ShardedCorpus.from_assignments(docs, assign, 2, 5)
    assert c.token_counts == {0: 40, 1: 40} and c.doc_counts == {0: 4, 1: 4}
    assert c.shard_weight(0) == pytest.approx(0.5)
    lop = ShardedCorpus.from_assignments(docs, torch.tensor([0, 0, 0, 1]), 2, 5)
    assert lop.shard_weight(0) == pytest.approx(0.75)


def test_loss_based_assignment_matches_the_argmin_and_respects_candidates():
    cfg = tiny_config()
    e = engine(cfg)
    g = torch.Generator().manual_seed(0)
    with torch.no_grad():  # experts start identical: make the paths differ
        for m in e.bank.values():
            for p in m.parameters():
                p.add_(0.2 * torch.randn(p.shape, generator=g))
    docs = banded_docs(cfg.backbone.vocab_size, per=3, length=20)
    losses = path_losses(docs, cfg, e.bank, 16, batch_size=5)
    assert losses.shape == (len(docs), cfg.num_paths) and torch.isfinite(losses).all()
    assert torch.equal(assign_paths_by_loss(docs, cfg, e.bank, 16, batch_size=5), losses.argmin(1))
    two = assign_paths_by_loss(docs, cfg, e.bank, 16, top_k=2)
    assert torch.equal(two[:, 0], losses.argmin(1)) and (two[:, 0] != two[:, 1]).all()
    only = path_losses(docs, cfg, e.bank, 16, candidates=[1, 3])
    assert torch.isinf(only[:, [0, 2]]).all() and torch.allclose(only[:, [1, 3]], losses[:, [1, 3]])
    corpus = reshard_by_loss(docs, cfg, e.bank, 16)
    want = {p: int((losses.argmin(1) == p).sum()) for p in range(cfg.num_paths)}
    assert corpus.doc_counts == want


# ------------------------------------------------------------------ memory estimator
def test_param_counts_and_breakdown_terms_are_exact():
    cfg = tiny_config(embedding="private", head="private")
    total, private, emb, head = _count_params(cfg)
    e = engine(cfg)
    path = e.topology.path_from_index(0)
    keys = e.topology.path_module_keys(path)
    assert total == sum(p.numel() for k in keys for p in e.bank[k].parameters())
    assert private == sum(p.numel() for k in keys if k.startswith(("embed", "head")) for p in e.bank[k].parameters())
    bd = vram_breakdown(cfg, batch_size=4, seq_len=16)
    assert bd["params"] == 4 * total and bd["adam"] == 8 * total and bd["grads"] == 4 * total
    assert bd["total"] == bd["params"] + bd["global"] + bd["adam"] + bd["grads"] + bd["activations"]
    assert fits(bd, bd["total"]) and not fits(bd, bd["total"] - 1)


def test_memory_levers_reduce_the_estimate():
    cfg = tiny_config(hidden=64, vocab=512)
    base = vram_breakdown(cfg, batch_size=8, seq_len=64)
    for lever in (dict(autocast=True), dict(checkpoint=True), dict(chunked_logits=True), dict(master_bytes=2)):
        assert vram_breakdown(cfg, batch_size=8, seq_len=64, **lever)["total"] < base["total"], lever


# ------------------------------------------------------------------ shard cache
def test_shard_cache_is_lru_and_validated():
    c = ShardCache(2)
    c[(0, 0)], c[(0, 1)] = torch.zeros(1), torch.ones(1)
    _ = c[(0, 0)]                 # a read marks it most recently used
    c[(1, 0)] = torch.full((1,), 2.0)
    assert list(c) == [(0, 0), (1, 0)]
    one = ShardCache(1)
    for _ in range(3):
        one[(0, 0)] = torch.zeros(1)  # a one-path worker never evicts its own shard
    assert list(one) == [(0, 0)]
    assert ShardCache(None).maxsize == 4
    with pytest.raises(ValueError):
        ShardCache(0)
