"""Data pipeline, path models and routed evaluation on CPU: tokenization rules, the
tokenizer trainer, deterministic splits, packing modes, identical-expert init, the
causal path model, and routed / windowed perplexity.

Behaviours of the reference's ``tests/test_data_pipeline.py``, ``tests/test_init_packing.py``,
``tests/test_model.py`` and ``tests/test_inference.py``.
"""

import math

import pytest
import torch

from opendipaco_b200.data import ShardedCorpus
from opendipaco_b200.data.sharding import chunk_documents, pack_sequences
from opendipaco_b200.data.text import split_documents, tokenize_documents, train_tokenizer
from opendipaco_b200.inference import compose_path, perplexity, routed_perplexity, routed_window_perplexity
from opendipaco_b200.models.path import build_module_bank, build_path_model

from helpers import tiny_config


class _WordTok:
    eos_token_id = 1

    def encode(self, text, add_special_tokens=False):
        return [2 + len(w) for w in text.split()]


# ------------------------------------------------------------------ tokenization
def test_tokenization_eos_truncation_and_filters():
    docs = tokenize_documents(["a bb ccc", "dddd"], _WordTok())
    assert [d.tolist() for d in docs] == [[3, 4, 5, 1], [6, 1]] and all(d.dtype == torch.long for d in docs)
    assert [d.tolist() for d in tokenize_documents(["a bb ccc"], _WordTok(), add_eos=False)] == [[3, 4, 5]]
    assert tokenize_documents(["a bb ccc dd"], _WordTok(), max_doc_tokens=3)[0].tolist() == [3, 4, 1]
    assert tokenize_documents(["a", "a bb ccc"], _WordTok(), min_doc_tokens=3)[0].tolist() == [3, 4, 5, 1]


def test_trained_tokenizers_round_trip_and_feed_a_corpus():
    texts = [f"the cat {w} sat on the mat {i}" for i, w in enumerate(["red", "blue", "green", "gray"] * 20)]
    for model in ("unigram", "bpe"):
        tok = train_tokenizer(texts, vocab_size=120, model=model)
        ids = tok.encode("the cat sat", add_special_tokens=False)
        assert tok.decode(ids).strip() == "the cat sat"
        docs = tokenize_documents(texts, tok)
        c = ShardedCorpus.from_assignments(docs, torch.arange(len(docs)) % 2, 2, 8)
        assert c.shard(0).size(1) == 8 and int(c.shard(0).max()) < len(tok)
    with pytest.raises(ValueError):
        train_tokenizer(texts, model="wordpiece")


def test_split_is_deterministic_and_partitions():
    docs = [torch.tensor([i]) for i in range(50)]
    tr, va, te = split_documents(docs, val_fraction=0.2, test_fraction=0.1, seed=3)
    again = split_documents(docs, val_fraction=0.2, test_fraction=0.1, seed=3)
    assert [len(x) for x in (tr, va, te)] == [35, 10, 5]
    assert all([a.item() for a in x] == [b.item() for b in y] for x, y in zip((tr, va, te), again))
    assert sorted(int(d) for part in (tr, va, te) for d in part) == list(range(50))


# ------------------------------------------------------------------ packing and init
def test_document_windows_never_span_two_documents():
    docs = [torch.arange(10), torch.arange(100, 107), torch.arange(200, 212)]
    chunks = chunk_documents(docs, 4)
    assert chunks.tolist() == [[0, 1, 2, 3], [4, 5, 6, 7], [100, 101, 102, 103], [200, 201, 202, 203],
                               [204, 205, 206, 207], [208, 209, 210, 211]]
    packed = pack_sequences(docs, 4)
    assert packed.size(0) == 29 // 4 and packed[2].tolist() == [8, 9, 100, 101]
    c = ShardedCorpus.from_assignments(docs, torch.zeros(3, dtype=torch.long), 1, 4, pack_mode="document")
    assert torch.equal(c.shard(0), chunks)
    with pytest.raises(ValueError):
        ShardedCorpus.from_assignments(docs, torch.zeros(3, dtype=torch.long), 1, 4, pack_mode="zip")


def test_experts_start_identical_unless_disabled():
    cfg = tiny_config(embedding="private", head="private")
    bank = build_module_bank(cfg, seed=0)
    for a, b in (("L0E0", "L0E1"), ("L1E0", "L1E1"), ("embed.p0", "embed.p3"), ("head.p1", "head.p2")):
        assert all(torch.equal(x, y) for x, y in zip(bank[a].parameters(), bank[b].parameters())), (a, b)
    cfg.identical_expert_init = False
    free = build_module_bank(cfg, seed=0)
    assert not all(torch.equal(x, y) for x, y in zip(free["L0E0"].parameters(), free["L0E1"].parameters()))


# ------------------------------------------------------------------ path model
def test_path_model_shapes_causality_and_copies():
    cfg = tiny_config()
    bank = build_module_bank(cfg, seed=0)
    topo = cfg.build_topology()
    path = topo.path_from_index(3)
    model = build_path_model(cfg, path, bank).eval()
    ids = torch.randint(0, 48, (2, 12))
    logits, _ = model(ids)
    assert logits.shape == (2, 12, 48)
    changed = ids.clone()
    changed[:, 7:] = (changed[:, 7:] + 1) % 48  # the future changes; the past's logits do not
    torch.testing.assert_close(model(changed)[0][:, :7], logits[:, :7])
    assert set(model.modules_by_key()) == set(topo.path_module_keys(path))
    copy = build_path_model(cfg, path, bank, deepcopy=True)
    with torch.no_grad():
        next(iter(copy.parameters())).add_(1.0)
    assert not torch.equal(next(iter(copy.parameters())), next(iter(bank[topo.path_module_keys(path)[0]].parameters())))


# ------------------------------------------------------------------ routed evaluation
class _Const:
    def __init__(self, p):
        self.p = p

    def predict(self, feats):
        return torch.full((feats.shape[0],), self.p, dtype=torch.long)


class _ByFirstToken:
    """Routes by the parity of the first token of the prefix (a stand-in for topics)."""

    def predict(self, feats):
        return (feats[:, 0] % 2).long()


def _first_token(prefixes):
    return torch.stack([p[:1].float() for p in prefixes])


def test_routed_perplexity_is_token_level_and_skips_the_routing_prefix():
    cfg = tiny_config()
    bank = build_module_bank(cfg, seed=0)
    seqs = torch.randint(0, 48, (6, 20), generator=torch.Generator().manual_seed(1))
    ppl = routed_perplexity(cfg, bank, seqs, _Const(2), _first_token, prefix_len=5)
    model = compose_path(cfg, bank, cfg.build_topology().path_from_index(2)).eval()
    with torch.no_grad():
        logits, _ = model(seqs)
        ce = torch.nn.functional.cross_entropy(logits[:, 4:-1].reshape(-1, 48), seqs[:, 5:].reshape(-1))
    assert ppl == pytest.approx(math.exp(ce.item()), rel=1e-5)
    assert math.isfinite(perplexity(model, seqs))


def test_windowed_evaluation_matches_one_path_and_reroutes_on_a_topic_shift():
    cfg = tiny_config()
    bank = build_module_bank(cfg, seed=0)
    with torch.no_grad():  # make paths 0 and 1 differ
        for p in bank["L1E1"].parameters():
            p.add_(0.3 * torch.randn(p.shape, generator=torch.Generator().manual_seed(2)))
    seqs = torch.randint(0, 48, (4, 24), generator=torch.Generator().manual_seed(3))
    one = routed_window_perplexity(cfg, bank, seqs, _Const(1), _first_token, window=24, prefix_len=4)
    assert one == pytest.approx(routed_perplexity(cfg, bank, seqs, _Const(1), _first_token, prefix_len=4), rel=1e-5)
    shifted = torch.randint(0, 48, (4, 36), generator=torch.Generator().manual_seed(4))
    shifted[:, 0] = 0   # even first token: windows 0 and 1 (routed by window 0) go to path 0
    shifted[:, 12] = 1  # odd start of window 1: window 2 (routed by window 1) goes to path 1
    r = routed_window_perplexity(cfg, bank, shifted, _ByFirstToken(), _first_token, window=12, prefix_len=4)
    p0 = routed_window_perplexity(cfg, bank, shifted, _Const(0), _first_token, window=12, prefix_len=4)
    assert math.isfinite(r) and r != pytest.approx(p0, rel=1e-6)


@pytest.mark.parametrize("window,prefix", [(12, 4), (7, 10), (16, 0), (50, 4)])
def test_cached_windowed_evaluation_equals_recomputing_the_prefix(window, prefix):
    cfg = tiny_config(heads=4, kv=2)
    bank = build_module_bank(cfg, seed=0)
    with torch.no_grad():
        for k in ("L1E1", "L0E1"):
            for p in bank[k].parameters():
                p.add_(0.3 * torch.randn(p.shape, generator=torch.Generator().manual_seed(2)))

    class _Mod4:
        def predict(self, feats):
            return (feats[:, 0] % 4).long()

    seqs = torch.randint(0, 48, (5, 50), generator=torch.Generator().manual_seed(3))
    cached = routed_window_perplexity(cfg, bank, seqs, _Mod4(), _first_token, window=window, prefix_len=prefix,
                                      batch_size=2)
    again = routed_window_perplexity(cfg, bank, seqs, _Mod4(), _first_token, window=window, prefix_len=prefix,
                                     batch_size=2, kv_cache=False)
    assert cached == pytest.approx(again, rel=1e-5)
