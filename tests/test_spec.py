"""Shard specs (data/spec.py): a recipe built here materializes to the same bytes and
fingerprint in the reference and vice versa, equals the shard a server would have sent,
routing is reproducible and verified once per recipe, a tampered router is refused, the
cache outlives the source, and C4 rows are budgeted and filtered (the behaviours of the
reference's tests/test_data_spec.py)."""

import pytest
import torch

from opendipaco_b200.data import spec as S


def _spec(mod, routing="kmeans"):
    src = mod.synthetic_source(vocab_size=512, num_documents=96, doc_len=80, topics=4, seed=3)
    if routing == "kmeans":
        r = mod.fit_routing_from_source(src, num_paths=4, vocab_size=512, seq_len=32, sample=64, feature_dim=32,
                                        router_seed=1, feat_seed=2)
    else:
        r = mod.round_robin_routing()
    return mod.make_shard_spec(source=src, routing=r, num_paths=4, seq_len=32, pack_mode="pack", prefix_len=16)


@pytest.mark.parametrize("routing", ["kmeans", "round_robin"])
def test_same_bytes_as_reference(routing, reference_pkg, tmp_path):
    from opendipaco.data import spec as R

    ours, theirs = _spec(S, routing), _spec(R, routing)
    # same recipe object -> same fingerprint; each framework's own fit agrees to float
    # rounding (the featurizers sum in different orders) and passes the other's check
    assert S.spec_fingerprint(ours) == R.spec_fingerprint(ours)
    if routing == "kmeans":
        torch.testing.assert_close(ours["routing"]["centroids"], theirs["routing"]["centroids"], rtol=1e-5, atol=1e-6)
        assert S.verify_routing(theirs) and R.verify_routing(ours)
    for p in range(4):
        a = S.materialize_shard(ours, p, cache_dir=tmp_path)
        b = R.materialize_shard(ours, p)
        assert torch.equal(a, b)
        assert torch.equal(S.materialize_shard(ours, p, cache_dir=tmp_path), a)  # from the cache file
    assert S.SpecCorpus.build(ours).token_counts == R.SpecCorpus.build(ours).token_counts


def test_verification_refuses_a_tampered_router():
    spec = _spec(S)
    assert S.verify_routing(spec)
    bad = dict(spec, routing=dict(spec["routing"], centroids=spec["routing"]["centroids"].flip(0)))
    assert not S.verify_routing(bad)
    assert S.spec_fingerprint(bad) != S.spec_fingerprint(spec)
    with pytest.raises(ValueError):
        S.make_shard_spec(source=spec["source"], routing=spec["routing"], num_paths=4, seq_len=32, pack_mode="zip")


# ------------------------------------------------------------------ sources and packing
def test_synthetic_documents_are_deterministic_and_banded():
    a = S.synthetic_documents(vocab_size=100, num_documents=12, doc_len=20, topics=4, seed=7)
    b = S.synthetic_documents(vocab_size=100, num_documents=12, doc_len=20, topics=4, seed=7)
    assert len(a) == 12 and all(torch.equal(x, y) for x, y in zip(a, b))
    for t in range(4):  # topic t's three documents use ids of its band only
        for d in a[3 * t:3 * t + 3]:
            assert int(d.min()) >= 25 * t and int(d.max()) < 25 * (t + 1)
    c = S.synthetic_documents(vocab_size=100, num_documents=12, doc_len=20, topics=4, seed=8)
    assert not all(torch.equal(x, y) for x, y in zip(a, c))


@pytest.mark.parametrize("routing", ["kmeans", "round_robin"])
@pytest.mark.parametrize("pack_mode", ["pack", "document"])
def test_materialized_shards_equal_the_server_side_corpus(routing, pack_mode):
    """A worker's shard from the recipe equals the shard a server would have built from
    the same documents and routing (and shipped as bytes)."""
    from opendipaco_b200.data import ShardedCorpus

    spec = dict(_spec(S, routing), pack_mode=pack_mode)
    docs, paths = zip(*S.iter_assignments(spec, None))
    corpus = ShardedCorpus.from_assignments(list(docs), torch.tensor(paths), 4, 32, pack_mode=pack_mode)
    for p in range(4):
        assert torch.equal(S.materialize_shard(spec, p), corpus.shard(p))


def test_spec_corpus_counts_tokens_per_path_and_holds_no_bytes():
    spec = _spec(S)
    sc = S.SpecCorpus.build(spec)
    totals = dict.fromkeys(range(4), 0)
    for d, p in S.iter_assignments(spec, None):
        totals[p] += d.numel()
    assert sc.token_counts == totals and sum(totals.values()) == 96 * 80
    assert abs(sum(sc.shard_weight(p) for p in range(4)) - 1.0) < 1e-9
    assert not sc.has_validation and sc.val_shard(0) is None
    with pytest.raises(RuntimeError):
        sc.shard(0)
    docs = list(S.iter_spec_documents(spec))
    assert S.SpecCorpus.from_documents(spec, docs).token_counts == totals
    with pytest.raises(ValueError):
        S.materialize_shard(spec, 4)


# ------------------------------------------------------------------ routing fits
def test_router_fit_is_deterministic_and_sample_bounded():
    src = S.synthetic_source(vocab_size=512, num_documents=96, doc_len=80, topics=4, seed=3)
    kw = dict(num_paths=4, vocab_size=512, seq_len=32, feature_dim=32, router_seed=1, feat_seed=2)
    a, b = S.fit_routing_from_source(src, sample=64, **kw), S.fit_routing_from_source(src, sample=64, **kw)
    assert torch.equal(a["centroids"], b["centroids"]) and a["fit"] == {"sample": 64, "router_seed": 1}
    # fewer sampled documents than paths: round-robin
    assert S.fit_routing_from_source(src, sample=3, **kw) == S.round_robin_routing()
    with pytest.raises(ValueError):
        S.fit_routing_from_source(src, sample=0, **kw)
    # a sample covering the corpus is the fit over every document's prefix
    from opendipaco_b200.routing.base import BagOfTokensFeaturizer
    from opendipaco_b200.routing.kmeans import KMeansRouter

    full = S.fit_routing_from_source(src, sample=10 ** 6, **kw)
    docs = S.synthetic_documents(vocab_size=512, num_documents=96, doc_len=80, topics=4, seed=3)
    feats = BagOfTokensFeaturizer(512, feature_dim=32, seed=2)([d[:32] for d in docs])
    torch.testing.assert_close(full["centroids"], KMeansRouter(4, seed=1).fit(feats).centroids)


def test_verification_covers_every_kind_of_tampering_and_its_limits():
    spec = _spec(S)
    r = spec["routing"]
    seed_swapped = dict(spec, routing=dict(r, featurizer=dict(r["featurizer"], seed=r["featurizer"]["seed"] + 1)))
    assert not S.verify_routing(seed_swapped)
    assert S.verify_routing(_spec(S, "round_robin"))  # nothing to check
    with pytest.raises(ValueError):  # no fit metadata: cannot be re-fitted
        S.verify_routing(dict(spec, routing={k: v for k, v in r.items() if k != "fit"}))
    with pytest.raises(ValueError):  # a featurizer kind nobody can re-run
        S.verify_routing(dict(spec, routing=dict(r, featurizer=dict(r["featurizer"], kind="model"))))
    with pytest.raises(ValueError):
        S.verify_routing(dict(spec, routing={"kind": "learned"}))
    # the source shrank below the path count: the re-fit degrades to round-robin
    tiny = dict(spec, source=dict(spec["source"], num_documents=2, topics=1))
    with pytest.raises(ValueError):
        S.verify_routing(tiny)


def test_worker_materialization_verifies_once_per_recipe(monkeypatch):
    from opendipaco_b200.schedule import distributed as D

    spec = _spec(S)
    calls = []
    real = D.verify_routing
    monkeypatch.setattr(D, "verify_routing", lambda *a, **k: calls.append(1) or real(*a, **k))
    ctx = {"verify": True}
    a = D.materialize_shard_spec({"spec": spec, "path_index": 1}, ctx)
    b = D.materialize_shard_spec({"spec": spec, "path_index": 2}, ctx)
    assert len(calls) == 1 and a.size(1) == b.size(1) == 32
    bad = dict(spec, routing=dict(spec["routing"], centroids=spec["routing"]["centroids"].flip(0)))
    with pytest.raises(D.RoutingVerificationError):
        D.materialize_shard_spec({"spec": bad, "path_index": 0}, ctx)
    # a recipe that cannot be verified (no fit metadata) proceeds with a warning
    nofit = dict(spec, routing={k: v for k, v in spec["routing"].items() if k != "fit"})
    assert torch.equal(D.materialize_shard_spec({"spec": nofit, "path_index": 1}, ctx), a)


def test_fingerprint_tracks_content_not_key_order():
    spec = _spec(S)
    fp = S.spec_fingerprint(spec)
    assert fp == S.spec_fingerprint(dict(reversed(list(spec.items())))) and len(fp) == 16
    for change in (dict(seq_len=64), dict(prefix_len=8), dict(num_paths=3), dict(pack_mode="document")):
        assert S.spec_fingerprint(dict(spec, **change)) != fp
    moved = spec["routing"]["centroids"].clone()
    moved[0, 0] += 1e-3
    assert S.spec_fingerprint(dict(spec, routing=dict(spec["routing"], centroids=moved))) != fp


def test_cached_shard_survives_loss_of_the_source(tmp_path):
    """Once materialized with a cache directory, a shard is read back even when the
    source can no longer be streamed (an offline worker)."""
    texts = [{"text": "alpha beta gamma delta " * (i + 2)} for i in range(12)]

    class Tok:
        eos_token_id = 0

        def encode(self, text, add_special_tokens=False):
            return [1 + (hash(w) % 50) for w in text.split()]

    src = S.c4_source(num_documents=12, tokenizer="fake", max_doc_tokens=20, min_doc_tokens=5)
    spec = S.make_shard_spec(source=src, routing=S.round_robin_routing(), num_paths=2, seq_len=8)
    tok = Tok()
    a = S.materialize_shard(spec, 1, source=iter(texts), tokenizer=tok, cache_dir=tmp_path)

    def gone():
        raise OSError("source offline")
        yield  # noqa: unreachable

    assert torch.equal(S.materialize_shard(spec, 1, source=gone(), tokenizer=tok, cache_dir=tmp_path), a)


def test_c4_source_honours_the_row_budget_and_length_filters():
    class Tok:
        eos_token_id = 99

        def encode(self, text, add_special_tokens=False):
            return [len(w) for w in text.split()]

    rows = ["a", "bb cc", "d e f g h i j k l m n", "x y z"] * 3
    src = S.c4_source(num_documents=4, tokenizer="fake", max_doc_tokens=6, min_doc_tokens=3)
    spec = S.make_shard_spec(source=src, routing=S.round_robin_routing(), num_paths=1, seq_len=4)
    docs = list(S.iter_spec_documents(spec, source=iter(rows), tokenizer=Tok()))
    # 4 rows read (the budget), "a" (2 tokens with EOS) filtered out, the long row capped at 6
    assert [d.tolist() for d in docs] == [[2, 2, 99], [1, 1, 1, 1, 1, 99], [1, 1, 1, 99]]
