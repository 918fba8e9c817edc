"""Run a few eager fused inner steps of the headline workload, for kernel profiling.

    python -m opendipaco_b200.utils.profile_step --paths 16 --rounds 2 --inner-steps 1

builds the 16-path hidden-384 DiPaCo (vocab 32000, seq 128, batch 24 per path) with
the given number of paths on one GPU, and runs ``rounds`` rounds of ``inner_steps``
inner steps without CUDA graphs, so a kernel profiler sees every launch. The first
round is the warm-up; with ``--inner-steps 1`` the second round is exactly one inner
step + one outer step (102 + 1 kernel launches for 4 layers).
"""

from __future__ import annotations

import argparse

import torch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--paths", type=int, default=16)
    ap.add_argument("--rounds", type=int, default=2)
    ap.add_argument("--inner-steps", type=int, default=1)
    ap.add_argument("--hidden", type=int, default=384)
    ap.add_argument("--heads", type=int, default=6)
    ap.add_argument("--ffn", type=int, default=1024)
    ap.add_argument("--vocab", type=int, default=32000)
    ap.add_argument("--seq", type=int, default=128)
    ap.add_argument("--batch", type=int, default=24)
    a = ap.parse_args(argv)

    from opendipaco_b200 import (BackboneConfig, DiLoCoConfig, DiPaCoConfig, DiPaCoEngine, ExecOptions,
                                 LocalBackend)
    from opendipaco_b200.data import ShardedCorpus, zipf_documents
    from opendipaco_b200.parallel.placement import rank_paths

    bb = BackboneConfig(vocab_size=a.vocab, hidden_size=a.hidden, num_attention_heads=a.heads,
                        intermediate_size=a.ffn, layers_per_level=[2, 2], max_position_embeddings=2048)
    cfg = DiPaCoConfig(backbone=bb, level_sizes=[4, 4], sequence_length=a.seq)
    dl = DiLoCoConfig(inner_steps=a.inner_steps, inner_autocast=True)
    topo = cfg.build_topology()

    class Subset(LocalBackend):
        def owned_paths(self):
            return [topo.path_from_index(i) for i in rank_paths(16, 16 // a.paths, 0)]

    docs = zipf_documents(vocab_size=a.vocab, num_documents=4000, min_len=128, max_len=2048, seed=0)
    corpus = ShardedCorpus.from_assignments(docs, torch.arange(len(docs)) % 16, 16, a.seq)
    eng = DiPaCoEngine(cfg, dl, Subset(topo), device="cuda", seed=0, exec_options=ExecOptions(cuda_graphs=False))
    for _ in range(a.rounds):
        eng.fit(corpus, num_rounds=1, batch_size=a.batch, log_every=0)
    torch.cuda.synchronize()
    print("ok")


if __name__ == "__main__":
    main()
