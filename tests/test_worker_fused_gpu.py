"""Workers on the B200 kernels: AsyncScheduler tasks (the body of asynchronous, sharded
and volunteer workers) trained by the fused one-path trainer against the PyTorch module
path, the speed-up, and a local coordinator run whose workers use it."""

import time

import pytest
import torch

from opendipaco_b200 import BackboneConfig, DiLoCoConfig, DiPaCoConfig, DiPaCoEngine, ExecOptions, LocalBackend
from opendipaco_b200.data import ShardedCorpus, zipf_documents
from opendipaco_b200.schedule import AsyncScheduler

pytestmark = pytest.mark.gpu


def _setup(layers=(1, 1), inner_steps=4):
    bb = BackboneConfig(vocab_size=512, hidden_size=128, num_attention_heads=2, intermediate_size=256,
                        layers_per_level=list(layers), max_position_embeddings=128)
    cfg = DiPaCoConfig(backbone=bb, level_sizes=[2, 2], sequence_length=64)
    docs = zipf_documents(vocab_size=512, num_documents=160, min_len=64, max_len=400, seed=1)
    corpus = ShardedCorpus.from_assignments(docs, torch.arange(len(docs)) % 4, 4, 64)
    dl = DiLoCoConfig(inner_steps=inner_steps, inner_lr=1e-3, inner_autocast=True)
    eng = DiPaCoEngine(cfg, dl, LocalBackend(cfg.build_topology()), device="cuda", seed=0, materialize="serial",
                       exec_options=ExecOptions(fused=False))
    return eng, corpus


def _bank(eng):
    return {k: {n: t.detach().float().cpu().clone() for n, t in m.state_dict().items()} for k, m in eng.bank.items()}


def test_fused_worker_tasks_track_the_module_path(monkeypatch):
    from opendipaco_b200.train.worker_trainer import FusedPathTrainer

    eng_a, corpus = _setup()
    eng_b, _ = _setup()
    before = FusedPathTrainer.tasks_trained
    ha = AsyncScheduler(eng_a, num_workers=2).fit(corpus, 2, 4, log_every=0)
    assert FusedPathTrainer.tasks_trained - before == 8  # 4 paths x 2 generations on the fused trainer
    monkeypatch.setenv("ODP_WORKER_FUSED", "0")
    hb = AsyncScheduler(eng_b, num_workers=2).fit(corpus, 2, 4, log_every=0)
    for a, b in zip(ha, hb):
        for p in b.per_path_loss:
            assert abs(a.per_path_loss[p] - b.per_path_loss[p]) < 3e-2 * b.per_path_loss[p], (p, a, b)
    ba, bb = _bank(eng_a), _bank(eng_b)
    worst = max((ba[k][n] - bb[k][n]).abs().max().item() for k in bb for n in bb[k])
    assert worst < 1.5e-2
    # the AdamW state persisted between generations carries the step count
    st = next(iter(eng_a._opt_state.values()))["state"]
    assert float(next(iter(st.values()))["step"]) == 8.0


def test_fused_worker_generation_is_faster(monkeypatch):
    eng_f, corpus = _setup(layers=(2, 2), inner_steps=10)
    eng_m, _ = _setup(layers=(2, 2), inner_steps=10)
    sf, sm = AsyncScheduler(eng_f, num_workers=1), AsyncScheduler(eng_m, num_workers=1)
    sf.fit(corpus, 1, 8, log_every=0)  # warm-up: arena, graph capture
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    sf.fit(corpus, 2, 8, log_every=0)
    torch.cuda.synchronize()
    fused_s = time.perf_counter() - t0
    monkeypatch.setenv("ODP_WORKER_FUSED", "0")
    sm.fit(corpus, 1, 8, log_every=0)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    sm.fit(corpus, 2, 8, log_every=0)
    torch.cuda.synchronize()
    module_s = time.perf_counter() - t0
    print(f"worker generations: fused {fused_s:.3f} s, module {module_s:.3f} s, {module_s / fused_s:.1f}x")
    assert module_s > 2.0 * fused_s, (fused_s, module_s)


def test_local_coordinator_run_trains_on_the_fused_kernels(tmp_path):
    from opendipaco_b200.launch.config import LaunchConfig
    from opendipaco_b200.launch.roles import run_local
    from opendipaco_b200.train.worker_trainer import FusedPathTrainer

    cfg = LaunchConfig.from_dict({
        "mode": "coordinator",
        "model": {"vocab_size": 512, "hidden_size": 128, "num_attention_heads": 2, "intermediate_size": 256,
                  "layers_per_level": [1, 1], "level_sizes": [2, 2], "sequence_length": 64,
                  "max_position_embeddings": 128},
        "diloco": {"inner_steps": 2, "inner_autocast": True, "activation_checkpoint": False},
        "data": {"num_documents": 64, "synthetic_doc_len": 160, "routing": "round_robin"},
        "transport": {"host": "127.0.0.1", "port": 0},
        "run": {"generations": 1, "batch_size": 2, "device": "cuda", "local_workers": 2}})
    before = FusedPathTrainer.tasks_trained
    server, completed = run_local(cfg)
    assert min(completed.values()) >= 1
    assert FusedPathTrainer.tasks_trained - before >= 4
