"""Worker for the multi-process tests (launched with torch.distributed.run).

    python -m torch.distributed.run --nproc-per-node N tests/mp_worker.py OUT_DIR MODE

MODE: "cpu" (gloo, module executor, TorchDistBackend), "nccl" (fused executor,
NCCL outer step) or "nvlink" (fused executor, peer-memory outer step); a "_dp2"
suffix puts every path on a group of two ranks (intra-path data parallelism), a further
"_8bit" suffix selects blockwise 8-bit Adam as the inner optimizer, and "nvlink_q4" sends
int4 codes instead of fp32 partials through the NVLink outer step ("nvlink_topk": the
top 5% of each 4096-element block as (index, value) pairs). Writes
``OUT_DIR/{MODE}_rank{r}.pt`` with the rank's bank, losses and a consistency flag.
"""

import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from opendipaco_b200 import (BackboneConfig, DiLoCoConfig, DiPaCoConfig, DiPaCoEngine, load_checkpoint,  # noqa
                             save_checkpoint)
from opendipaco_b200.data import ShardedCorpus, zipf_documents  # noqa: E402
from opendipaco_b200.parallel import TorchDistBackend  # noqa: E402
from opendipaco_b200.topology import is_private_key  # noqa: E402


def main():
    out_dir, mode = sys.argv[1], sys.argv[2]
    q4 = mode.endswith("_q4")
    topk = mode.endswith("_topk")
    rest = mode[:-3] if q4 else mode[:-5] if topk else mode
    opt8 = rest.endswith("_8bit")
    core = rest[:-5] if opt8 else rest
    dp = 2 if core.endswith("_dp2") else 1
    base = core[:-4] if dp > 1 else core
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    if base == "cpu":
        dist.init_process_group("gloo", timeout=timedelta(seconds=60))
        dev = torch.device("cpu")
        bb = BackboneConfig(vocab_size=128, hidden_size=32, num_attention_heads=4, intermediate_size=64,
                            layers_per_level=[1, 1], max_position_embeddings=64)
        seq = 16
    else:
        local = int(os.environ["LOCAL_RANK"])
        torch.cuda.set_device(local)
        dev = torch.device("cuda", local)
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=60))
        bb = BackboneConfig(vocab_size=512, hidden_size=128, num_attention_heads=2, intermediate_size=256,
                            layers_per_level=[1, 1], max_position_embeddings=128)
        seq = 64
    cfg = DiPaCoConfig(backbone=bb, level_sizes=[2, 2], sequence_length=seq)
    dl = DiLoCoConfig(inner_steps=3, inner_lr=1e-3, inner_autocast=base != "cpu", optim_8bit=opt8)
    docs = zipf_documents(vocab_size=bb.vocab_size, num_documents=160, min_len=64, max_len=400, seed=1)
    corpus = ShardedCorpus.from_assignments(docs, torch.arange(len(docs)) % 4, 4, seq)
    topo = cfg.build_topology()
    if base == "nvlink":
        from opendipaco_b200.parallel.backend.nvlink import NVLinkBackend

        backend = NVLinkBackend(topo, device=dev, dp=dp, compress="int4" if q4 else "topk" if topk else None,
                                density=0.05)
    else:
        backend = TorchDistBackend(topo, device=dev, dp=dp)
    eng = DiPaCoEngine(cfg, dl, backend, device=dev, seed=0)
    init = {k: {n: t.detach().cpu().clone() for n, t in m.state_dict().items()} for k, m in eng.bank.items()}
    hist = eng.fit(corpus, num_rounds=3, batch_size=4, log_every=0)
    # shared modules must be identical on every rank that owns them
    consistent = True
    for key in topo.module_keys():
        if is_private_key(key):
            continue
        owned = key in eng.bank
        flat = (torch.cat([p.detach().reshape(-1).float() for p in eng.bank[key].parameters()]) if owned
                else torch.zeros(1, device=dev))
        n = torch.tensor([flat.numel() if owned else 0], device=dev)
        gathered = [torch.zeros_like(n) for _ in range(world)]
        dist.all_gather(gathered, n)
        size = max(int(g.item()) for g in gathered)
        buf = torch.zeros(size, device=dev)
        if owned:
            buf.copy_(flat)
        allb = [torch.zeros_like(buf) for _ in range(world)]
        dist.all_gather(allb, buf)
        ranks = backend.sharing_ranks(key)
        for r in ranks[1:]:
            consistent &= bool(torch.equal(allb[r], allb[ranks[0]]))
    # full-bank gather: the NVLink pull equals the per-parameter broadcast bit for bit
    gather_same = True
    if base == "nvlink" and dp == 1:
        from opendipaco_b200.parallel.gather import gather_full_bank

        fb_peer = gather_full_bank(backend, eng.bank, cfg, method="peer")
        fb_bc = gather_full_bank(backend, eng.bank, cfg, method="broadcast")
        gather_same = sorted(fb_peer) == sorted(topo.module_keys()) and all(
            torch.equal(a, b) for k in fb_peer
            for a, b in zip(fb_peer[k].state_dict().values(), fb_bc[k].state_dict().values()))
    # checkpoint round trip (momentum gathered from the slice owners)
    ck = os.path.join(out_dir, f"ckpt_{mode}")
    save_checkpoint(eng, ck)
    b2 = (NVLinkBackend(topo, device=dev, dp=dp, compress="int4" if q4 else "topk" if topk else None,
                                density=0.05) if base == "nvlink"
          else TorchDistBackend(topo, device=dev, dp=dp))
    eng2 = DiPaCoEngine(cfg, dl, b2, device=dev, seed=5)
    load_checkpoint(eng2, ck)
    same = all(torch.equal(a, b) for k in eng.bank
               for a, b in zip(eng.bank[k].state_dict().values(), eng2.bank[k].state_dict().values()))
    h1 = eng.fit(corpus, num_rounds=1, batch_size=4, log_every=0)
    h2 = eng2.fit(corpus, num_rounds=1, batch_size=4, log_every=0)
    resumed = h1[0].per_path_loss == h2[0].per_path_loss
    torch.save({"bank": {k: {n: t.detach().cpu() for n, t in m.state_dict().items()} for k, m in eng.bank.items()},
                "init": init, "losses": [m.per_path_loss for m in hist], "consistent": consistent, "ckpt_same": same,
                "gather_same": gather_same, "resumed": resumed},
               os.path.join(out_dir, f"{mode}_rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
