"""Grouped multi-path scoring (EM losses, routed perplexity) against the path-by-path
module forward."""

import pytest
import torch

from opendipaco_b200 import BackboneConfig, DiPaCoConfig
from opendipaco_b200.data import zipf_documents
from opendipaco_b200.models.path import build_module_bank
from opendipaco_b200.train import scorer as SC

pytestmark = pytest.mark.gpu


def _setup(levels=(2, 2), kv=None, vocab=512):
    bb = BackboneConfig(vocab_size=vocab, hidden_size=128, num_attention_heads=2, num_key_value_heads=kv,
                        intermediate_size=256, layers_per_level=[1, 1], max_position_embeddings=256)
    cfg = DiPaCoConfig(backbone=bb, level_sizes=list(levels), sequence_length=128)
    bank = build_module_bank(cfg, seed=0)
    g = torch.Generator().manual_seed(5)
    with torch.no_grad():
        for mod in bank.values():  # make the experts differ
            for p in mod.parameters():
                p.add_(torch.randn(p.shape, generator=g) * 0.05)
    bank = {k: m.cuda() for k, m in bank.items()}
    return cfg, bank


def _module_path(monkeypatch):
    monkeypatch.setattr(SC.GroupedScorer, "supported", staticmethod(lambda *a: False))


def test_em_path_losses_grouped_match_module_forward(monkeypatch):
    from opendipaco_b200 import em

    cfg, bank = _setup()
    docs = zipf_documents(vocab_size=512, num_documents=37, min_len=20, max_len=150, seed=3)
    grouped = em.path_losses(docs, cfg, bank, seq_len=128, candidates=[0, 2, 3], batch_size=8)
    with monkeypatch.context() as m:
        _module_path(m)
        ref = em.path_losses(docs, cfg, bank, seq_len=128, candidates=[0, 2, 3], batch_size=8)
    assert torch.isinf(grouped[:, 1]).all() and torch.isinf(ref[:, 1]).all()
    fin = torch.isfinite(ref)
    assert torch.allclose(grouped[fin], ref[fin], rtol=0, atol=3e-2)
    best_g, best_r = grouped.min(1), ref.min(1)
    srt = ref.sort(1).values
    clear = (srt[:, 1] - srt[:, 0]) > 0.1
    assert torch.equal(best_g.indices[clear], best_r.indices[clear])


def test_routed_perplexity_grouped_matches_module_forward(monkeypatch):
    from opendipaco_b200.inference import routed_perplexity
    from opendipaco_b200.routing import BagOfTokensFeaturizer, KMeansRouter

    cfg, bank = _setup(kv=1)
    docs = zipf_documents(vocab_size=512, num_documents=90, min_len=200, max_len=300, seed=4)
    seqs = torch.stack([d[:160] for d in docs])
    feat = BagOfTokensFeaturizer(512, feature_dim=64, seed=0)
    router = KMeansRouter(4, seed=0).fit(feat([s[:32] for s in seqs]))
    ppl = routed_perplexity(cfg, bank, seqs, router, feat, prefix_len=32, batch_size=8)
    with monkeypatch.context() as m:
        _module_path(m)
        ref = routed_perplexity(cfg, bank, seqs, router, feat, prefix_len=32, batch_size=8)
    assert abs(ppl - ref) / ref < 2e-2


def test_grouped_scorer_rows_are_independent():
    """A group's losses do not depend on what the other groups hold."""
    cfg, bank = _setup()
    topo = cfg.build_topology()
    sc = SC.GroupedScorer(cfg, bank, torch.device("cuda"), groups=3, batch=2, seq_len=64)
    for g in range(3):
        sc.load(g, topo.path_from_index(g))
    ids = torch.randint(0, 512, (3, 2, 64), generator=torch.Generator().manual_seed(0)).cuda()
    tgt = torch.roll(ids, -1, dims=2)
    tgt[..., -1] = -100
    a = sc.token_losses(ids, tgt)
    ids2 = ids.clone()
    ids2[1] = torch.randint(0, 512, (2, 64), generator=torch.Generator().manual_seed(1)).cuda()
    sc.load(2, topo.path_from_index(3))
    b = sc.token_losses(ids2, tgt)
    assert torch.equal(a[0], b[0])
    assert (a[..., -1] == 0).all()
