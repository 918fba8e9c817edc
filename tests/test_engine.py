import torch

from opendipaco_b200 import DiLoCoConfig, DiPaCoEngine, LocalBackend
from opendipaco_b200.routing import BagOfTokensFeaturizer, KMeansRouter
from opendipaco_b200.data import ShardedCorpus
from opendipaco_b200.topology import embed_key, expert_key, is_private_key
from opendipaco_b200.train.loop import _iter_batches, batch_indices

from helpers import banded_docs, engine, rr_corpus, tiny_config


def test_batches_without_replacement_within_epoch():
    shard = torch.arange(12).reshape(12, 1)
    bs = list(_iter_batches(shard, 4, 3, torch.Generator().manual_seed(0)))
    assert sorted(torch.cat([b.reshape(-1) for b in bs]).tolist()) == list(range(12))


def test_batches_continue_across_epochs():
    idx = batch_indices(6, 4, 5, torch.Generator().manual_seed(0))
    assert len(idx) == 5 and all(i.numel() == 4 for i in idx)


def _routed_setup(embedding="shared"):
    cfg = tiny_config(hidden=48, vocab=64, ffn=96, seq=32, embedding=embedding)
    docs = banded_docs(64, per=40, length=50)
    feat = BagOfTokensFeaturizer(64, feature_dim=64)
    router = KMeansRouter(cfg.num_paths, seed=0).fit(feat([d[:32] for d in docs]))
    return cfg, ShardedCorpus.from_documents(docs, router, feat, cfg.num_paths, 32)


def test_training_reduces_loss():
    cfg, corpus = _routed_setup()
    eng = engine(cfg, inner_steps=5)
    hist = eng.fit(corpus, num_rounds=8, batch_size=8, log_every=0)
    assert hist[-1].inner_loss < hist[0].inner_loss


def test_serial_matches_eager():
    cfg, corpus = _routed_setup()
    a, b = engine(cfg, "eager", inner_steps=5), engine(cfg, "serial", inner_steps=5)
    a.fit(corpus, num_rounds=3, batch_size=8, log_every=0)
    b.fit(corpus, num_rounds=3, batch_size=8, log_every=0)
    assert not b.path_models and b._opt_state
    for k in a.bank:
        for x, y in zip(a.bank[k].parameters(), b.bank[k].parameters()):
            assert torch.allclose(x, y, atol=1e-5), k


def test_shared_synced_and_expert_isolation():
    cfg, corpus = _routed_setup()
    eng = engine(cfg, inner_steps=3)
    eng.run_round(corpus, batch_size=8)
    g = next(eng.bank[embed_key()].parameters())
    for pm in eng.path_models.values():
        assert torch.equal(next(pm.modules_by_key()[embed_key()].parameters()), g)
    e = next(eng.bank[expert_key(0, 0)].parameters())
    for path in [(0, 0), (0, 1)]:
        assert torch.equal(next(eng.path_models[path].modules_by_key()[expert_key(0, 0)].parameters()), e)


def test_private_embedding_diverges_and_not_outer_stepped():
    cfg, corpus = _routed_setup(embedding="private")
    eng = engine(cfg, inner_steps=5)
    assert "embed" not in eng.bank and "embed.p0" in eng.bank
    outer = {id(p) for g in eng.outer_opt.param_groups for p in g["params"]}
    for k, m in eng.bank.items():
        assert any(id(p) in outer for p in m.parameters()) == (not is_private_key(k))
    eng.run_round(corpus, batch_size=8)
    assert not torch.allclose(next(eng.bank["embed.p0"].parameters()),
                              next(eng.bank["embed.p3"].parameters()))


def test_empty_shard_is_skipped():
    cfg = tiny_config()
    docs = banded_docs(48)
    corpus = ShardedCorpus.from_assignments(docs, torch.zeros(len(docs), dtype=torch.long), 4, 16)
    eng = engine(cfg, inner_steps=2)
    m = eng.run_round(corpus, batch_size=4)
    assert list(m.per_path_loss) == [(0, 0)]


def test_matches_reference_engine_bitwise(reference_pkg):
    """Same seed + same data -> the reference's CPU engine and ours agree exactly."""
    R = reference_pkg
    from opendipaco.data import ShardedCorpus as RSC

    cfg = tiny_config(hidden=64, vocab=128, ffn=128, seq=32)
    rcfg = R.DiPaCoConfig(backbone=R.BackboneConfig(**vars(cfg.backbone)), level_sizes=[2, 2],
                          sequence_length=32)
    assert repr(rcfg) == repr(cfg)
    docs = banded_docs(128, per=16, length=100)
    assign = torch.arange(len(docs)) % 4
    dl = dict(inner_steps=3, inner_lr=1e-3)
    ours = DiPaCoEngine(cfg, DiLoCoConfig(**dl), LocalBackend(cfg.build_topology()), seed=3)
    ref = R.DiPaCoEngine(rcfg, R.DiLoCoConfig(**dl), R.LocalBackend(rcfg.build_topology()), seed=3)
    h1 = ours.fit(ShardedCorpus.from_assignments(docs, assign, 4, 32), 2, 8, log_every=0)
    h2 = ref.fit(RSC.from_assignments(docs, assign, 4, 32), 2, 8, log_every=0)
    assert [m.inner_loss for m in h1] == [m.inner_loss for m in h2]
    for k in ref.bank:
        for a, b in zip(ref.bank[k].state_dict().values(), ours.bank[k].state_dict().values()):
            assert torch.equal(a, b)


def test_routed_perplexity_matches_reference(reference_pkg):
    """Held-out routed perplexity: both frameworks train the same 2x2 DiPaCo on the same
    shards (bit-identical banks), route held-out documents with their own k-means router
    over their own bag-of-tokens featuriser, and score them with their own
    ``routed_perplexity`` -- the numbers are equal."""
    R = reference_pkg
    from opendipaco.data import ShardedCorpus as RSC
    from opendipaco.inference import routed_perplexity as r_ppl
    from opendipaco.routing import BagOfTokensFeaturizer as RBag, KMeansRouter as RKM

    from opendipaco_b200.inference import routed_perplexity
    from opendipaco_b200.routing import BagOfTokensFeaturizer, KMeansRouter

    cfg = tiny_config(hidden=64, vocab=128, ffn=128, seq=32)
    rcfg = R.DiPaCoConfig(backbone=R.BackboneConfig(**vars(cfg.backbone)), level_sizes=[2, 2],
                          sequence_length=32)
    docs = banded_docs(128, per=20, length=100)
    train, held = docs[::2], docs[1::2]
    feat, rfeat = BagOfTokensFeaturizer(128, feature_dim=32, seed=0), RBag(128, feature_dim=32, seed=0)
    router = KMeansRouter(4, seed=0).fit(feat([d[:16] for d in train]))
    rrouter = RKM(4, seed=0).fit(rfeat([d[:16] for d in train]))
    assign = router.predict(feat([d[:16] for d in train]))
    assert torch.equal(assign, rrouter.predict(rfeat([d[:16] for d in train])))
    dl = dict(inner_steps=3, inner_lr=1e-3)
    ours = DiPaCoEngine(cfg, DiLoCoConfig(**dl), LocalBackend(cfg.build_topology()), seed=3)
    ref = R.DiPaCoEngine(rcfg, R.DiLoCoConfig(**dl), R.LocalBackend(rcfg.build_topology()), seed=3)
    ours.fit(ShardedCorpus.from_assignments(train, assign, 4, 32), 3, 8, log_every=0)
    ref.fit(RSC.from_assignments(train, assign, 4, 32), 3, 8, log_every=0)
    seqs = torch.stack([d[:64] for d in held])
    p_ours = routed_perplexity(cfg, ours.global_modules(), seqs, router, feat, prefix_len=16)
    p_ref = r_ppl(rcfg, ref.global_modules(), seqs, rrouter, rfeat, prefix_len=16)
    assert p_ours == p_ref, (p_ours, p_ref)
    assert 1.0 < p_ours < float("inf")
