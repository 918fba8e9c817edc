"""DiPaCo vs. a matched dense baseline (reference ``src/opendipaco/validation.py``).

The dense baseline is DiPaCo with one expert per level (one path = one dense
model of the same size). Both train on the same documents; DiPaCo routes them with
k-means over ``ModelFeaturizer`` features, then a discriminative router is fit on
a held-out slice, and both are scored with ``routed_perplexity``.
"""

from __future__ import annotations

import torch

from .config import BackboneConfig, DiLoCoConfig, DiPaCoConfig
from .data import ShardedCorpus, pack_sequences
from .em import fit_discriminative_router
from .inference import routed_perplexity
from .parallel.backend import LocalBackend
from .routing import BagOfTokensFeaturizer, KMeansRouter, ModelFeaturizer
from .train import DiPaCoEngine


class _ZeroRouter:
    def predict(self, features) -> torch.Tensor:
        return torch.zeros(features.shape[0], dtype=torch.long)

    def predict_topk(self, features, k) -> torch.Tensor:
        return torch.zeros(features.shape[0], k, dtype=torch.long)


def _params(engine) -> int:
    return sum(p.numel() for m in engine.bank.values() for p in m.parameters())


def run_comparison(backbone: BackboneConfig, train_docs: list, test_docs: list,
                   diloco: DiLoCoConfig, *, dipaco_levels=(2, 2), dense_levels=(1, 1),
                   rounds: int = 20, batch_size: int = 8, seq_len: int = 64, eval_len: int = 128,
                   seed: int = 0, router_seed: int = 0, router_holdout: float = 0.15,
                   device="cpu") -> dict:
    dense_cfg = DiPaCoConfig(backbone=backbone, level_sizes=list(dense_levels),
                             sequence_length=seq_len, eval_sequence_length=eval_len)
    dip_cfg = DiPaCoConfig(backbone=backbone, level_sizes=list(dipaco_levels),
                           sequence_length=seq_len, eval_sequence_length=eval_len)
    test = pack_sequences(test_docs, dense_cfg.eval_seq_len)
    n_hold = max(1, int(len(train_docs) * router_holdout))
    router_docs, core = train_docs[:n_hold], train_docs[n_hold:]

    dense = DiPaCoEngine(dense_cfg, diloco, LocalBackend(dense_cfg.build_topology()), seed=seed,
                         device=device)
    dcorp = ShardedCorpus.from_assignments(core, torch.zeros(len(core), dtype=torch.long),
                                           dense_cfg.num_paths, seq_len)
    dense.total_rounds = rounds
    dense.fit(dcorp, num_rounds=rounds, batch_size=batch_size, log_every=0)
    dense_ppl = routed_perplexity(dense_cfg, dense.global_modules(), test, _ZeroRouter(),
                                  BagOfTokensFeaturizer(backbone.vocab_size))

    dip = DiPaCoEngine(dip_cfg, diloco, LocalBackend(dip_cfg.build_topology()), seed=seed,
                       device=device)
    feat = ModelFeaturizer(dip.global_modules(), dip_cfg, device=device)
    km = KMeansRouter(dip_cfg.num_paths, seed=router_seed).fit(feat([d[:seq_len] for d in core]))
    corp = ShardedCorpus.from_documents(core, km, feat, dip_cfg.num_paths, seq_len)
    dip.total_rounds = rounds
    dip.fit(corp, num_rounds=rounds, batch_size=batch_size, log_every=0)
    disc = fit_discriminative_router(router_docs, dip_cfg, dip.global_modules(), feat, seq_len)
    dip_ppl = routed_perplexity(dip_cfg, dip.global_modules(), test, disc, feat)
    return {"dense_ppl": dense_ppl, "dipaco_ppl": dip_ppl, "params_per_path": _params(dense),
            "dipaco_paths": dip_cfg.num_paths, "dipaco_total_params": _params(dip)}
