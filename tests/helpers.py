"""Small shared builders for the tests."""

import torch

from opendipaco_b200 import BackboneConfig, DiLoCoConfig, DiPaCoConfig, DiPaCoEngine, LocalBackend
from opendipaco_b200.data import ShardedCorpus


def tiny_config(levels=(2, 2), hidden=32, heads=4, vocab=48, ffn=64, seq=16, embedding="shared",
                head="shared", layers=None, kv=None):
    layers = list(layers or [1] * len(levels))
    bb = BackboneConfig(vocab_size=vocab, hidden_size=hidden, num_attention_heads=heads,
                        num_key_value_heads=kv, intermediate_size=ffn, layers_per_level=layers,
                        max_position_embeddings=max(64, seq))
    return DiPaCoConfig(backbone=bb, level_sizes=list(levels), sequence_length=seq,
                        embedding=embedding, head=head)


def banded_docs(vocab, n_topics=4, per=8, length=48, seed=0):
    g = torch.Generator().manual_seed(seed)
    span = vocab // n_topics
    return [torch.randint(t * span, (t + 1) * span, (length,), generator=g)
            for t in range(n_topics) for _ in range(per)]


def rr_corpus(cfg, docs=None, val_fraction=0.0):
    docs = docs if docs is not None else banded_docs(cfg.backbone.vocab_size)
    assign = torch.tensor([i % cfg.num_paths for i in range(len(docs))])
    return ShardedCorpus.from_assignments(docs, assign, cfg.num_paths, cfg.sequence_length,
                                          val_fraction=val_fraction)


def engine(cfg, materialize="eager", seed=0, **dl):
    d = dict(inner_steps=4, inner_lr=1e-3)
    d.update(dl)
    return DiPaCoEngine(cfg, DiLoCoConfig(**d), LocalBackend(cfg.build_topology()), seed=seed,
                        materialize=materialize)


def banks_equal(a, b):
    for k in a:
        pa, pb = dict(a[k].named_parameters()), dict(b[k].named_parameters())
        assert pa.keys() == pb.keys()
        if any(not torch.equal(pa[n], pb[n]) for n in pa):
            return False
    return True
