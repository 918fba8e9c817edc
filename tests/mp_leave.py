"""Worker of the rank-leaves test (launched with torch.distributed.run, 2 gloo ranks).

Both ranks train one synchronous round; then rank 1 leaves between rounds (no collective
of it in flight) and rank 0 starts the next round. Rank 0's first collective of that
round must end with an error within the short process-group timeout instead of hanging;
rank 0 records what it saw in OUT_DIR/leave_rank0.pt.
"""

import os
import sys
import time
from datetime import timedelta

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from opendipaco_b200 import BackboneConfig, DiLoCoConfig, DiPaCoConfig, DiPaCoEngine  # noqa: E402
from opendipaco_b200.data import ShardedCorpus, zipf_documents  # noqa: E402
from opendipaco_b200.parallel import TorchDistBackend  # noqa: E402


def main():
    out_dir = sys.argv[1]
    rank = int(os.environ["RANK"])
    dist.init_process_group("gloo", timeout=timedelta(seconds=5))
    bb = BackboneConfig(vocab_size=128, hidden_size=32, num_attention_heads=4, intermediate_size=64,
                        layers_per_level=[1, 1], max_position_embeddings=64)
    cfg = DiPaCoConfig(backbone=bb, level_sizes=[2, 2], sequence_length=16)
    docs = zipf_documents(vocab_size=128, num_documents=64, min_len=32, max_len=120, seed=1)
    corpus = ShardedCorpus.from_assignments(docs, torch.arange(len(docs)) % 4, 4, 16)
    eng = DiPaCoEngine(cfg, DiLoCoConfig(inner_steps=2, inner_lr=1e-3), TorchDistBackend(cfg.build_topology()),
                       seed=0)
    eng.fit(corpus, num_rounds=1, batch_size=2, log_every=0)
    if rank == 1:
        os._exit(0)  # leaves between rounds, without a goodbye
    time.sleep(1.0)
    t0 = time.monotonic()
    try:
        eng.fit(corpus, num_rounds=1, batch_size=2, log_every=0)
        outcome = {"detected": False}
    except Exception as exc:  # the next collective of the round fails
        outcome = {"detected": True, "error": repr(exc)[:300]}
    outcome["seconds"] = time.monotonic() - t0
    torch.save(outcome, os.path.join(out_dir, "leave_rank0.pt"))
    os._exit(0)


if __name__ == "__main__":
    main()
