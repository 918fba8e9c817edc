"""The fused B200 executor against the module executor (CPU oracle) and itself."""

import pytest
import torch

from opendipaco_b200 import (BackboneConfig, DiLoCoConfig, DiPaCoConfig, DiPaCoEngine, ExecOptions, LocalBackend,
                             load_checkpoint, save_checkpoint)
from opendipaco_b200.data import ShardedCorpus, zipf_documents

pytestmark = pytest.mark.gpu


def _cfg(embedding="shared", levels=(2, 2), layers=(1, 1), kv=None):
    bb = BackboneConfig(vocab_size=512, hidden_size=128, num_attention_heads=2, num_key_value_heads=kv,
                        intermediate_size=256, layers_per_level=list(layers), max_position_embeddings=128)
    return DiPaCoConfig(backbone=bb, level_sizes=list(levels), sequence_length=64, embedding=embedding)


def _corpus(cfg, n=160):
    docs = zipf_documents(vocab_size=512, num_documents=n, min_len=64, max_len=400, seed=1)
    a = torch.arange(len(docs)) % cfg.num_paths
    return ShardedCorpus.from_assignments(docs, a, cfg.num_paths, cfg.sequence_length)


def _engine(cfg, device, graphs=True, fused=None, **dl):
    d = dict(inner_steps=3, inner_lr=1e-3, inner_autocast=True)
    d.update(dl)
    return DiPaCoEngine(cfg, DiLoCoConfig(**d), LocalBackend(cfg.build_topology()), device=device, seed=0,
                        exec_options=ExecOptions(fused=fused, cuda_graphs=graphs))


def _bank_maxdiff(a, b):
    m = 0.0
    for k in a.bank:
        for x, y in zip(a.bank[k].state_dict().values(), b.bank[k].state_dict().values()):
            m = max(m, (x.float().cpu() - y.float().cpu()).abs().max().item())
    return m


def test_fused_matches_cpu_oracle():
    cfg = _cfg()
    corpus = _corpus(cfg)
    gpu = _engine(cfg, "cuda")
    assert gpu.fused
    cpu = _engine(cfg, "cpu")
    hg = gpu.fit(corpus, 3, 4, log_every=0)
    hc = cpu.fit(corpus, 3, 4, log_every=0)
    for a, b in zip(hg, hc):
        for p in a.per_path_loss:
            assert abs(a.per_path_loss[p] - b.per_path_loss[p]) < 3e-2 * b.per_path_loss[p], (p, a, b)
    assert _bank_maxdiff(gpu, cpu) < 1.5e-2


def test_graph_replay_equals_eager_bitwise():
    cfg = _cfg()
    corpus = _corpus(cfg)
    a, b = _engine(cfg, "cuda", graphs=True), _engine(cfg, "cuda", graphs=False)
    ha = a.fit(corpus, 4, 4, log_every=0)
    hb = b.fit(corpus, 4, 4, log_every=0)
    assert [m.per_path_loss for m in ha] == [m.per_path_loss for m in hb]
    assert _bank_maxdiff(a, b) == 0.0


def test_fused_resume_bit_for_bit(tmp_path):
    cfg = _cfg()
    corpus = _corpus(cfg)
    ref = _engine(cfg, "cuda")
    ref.fit(corpus, 4, 4, log_every=0, total_rounds=4)
    x = _engine(cfg, "cuda")
    x.fit(corpus, 2, 4, log_every=0, total_rounds=4)
    save_checkpoint(x, tmp_path / "c")
    y = _engine(cfg, "cuda")
    load_checkpoint(y, tmp_path / "c")
    y.fit(corpus, 2, 4, log_every=0)
    assert _bank_maxdiff(ref, y) == 0.0


def test_fused_checkpoint_loads_into_module_executor(tmp_path):
    cfg = _cfg()
    corpus = _corpus(cfg)
    g = _engine(cfg, "cuda")
    g.fit(corpus, 2, 4, log_every=0)
    save_checkpoint(g, tmp_path / "c")
    c = _engine(cfg, "cpu")
    load_checkpoint(c, tmp_path / "c")
    assert _bank_maxdiff(g, c) == 0.0
    st = c.inner_opts[(0, 0)].state_dict()["state"]
    assert st and float(next(iter(st.values()))["step"]) == 6


def test_fused_private_embedding_and_8bit():
    cfg = _cfg(embedding="private")
    corpus = _corpus(cfg)
    gpu = _engine(cfg, "cuda", optim_8bit=True)
    cpu = _engine(cfg, "cpu", optim_8bit=True)
    hg = gpu.fit(corpus, 2, 4, log_every=0)
    hc = cpu.fit(corpus, 2, 4, log_every=0)
    for a, b in zip(hg, hc):
        for p in a.per_path_loss:
            assert abs(a.per_path_loss[p] - b.per_path_loss[p]) < 3e-2 * b.per_path_loss[p]
    assert not torch.allclose(gpu.bank["embed.p0"].embed_tokens.weight, gpu.bank["embed.p3"].embed_tokens.weight)
    assert _bank_maxdiff(gpu, cpu) < 1e-2


def test_fused_gqa_and_deeper():
    cfg = _cfg(layers=(2, 1), kv=1, levels=(3, 2))
    corpus = _corpus(cfg, n=240)
    gpu, cpu = _engine(cfg, "cuda"), _engine(cfg, "cpu")
    hg, hc = gpu.fit(corpus, 2, 4, log_every=0), cpu.fit(corpus, 2, 4, log_every=0)
    for p in hg[-1].per_path_loss:
        assert abs(hg[-1].per_path_loss[p] - hc[-1].per_path_loss[p]) < 3e-2 * hc[-1].per_path_loss[p]


def test_module_forward_on_cuda_kernels_matches_cpu():
    from opendipaco_b200.models import build_path_model
    from opendipaco_b200.models.path import build_module_bank

    cfg = _cfg()
    torch.manual_seed(0)
    bank = build_module_bank(cfg)
    pm_c = build_path_model(cfg, (0, 1), bank, deepcopy=True)
    pm_g = build_path_model(cfg, (0, 1), bank, deepcopy=True).cuda()
    ids = torch.randint(0, 512, (3, 96))
    lc, loss_c = pm_c(ids, labels=ids)
    lg, loss_g = pm_g(ids.cuda(), labels=ids.cuda())
    assert abs(loss_c.item() - loss_g.item()) < 2e-2 * loss_c.item()
    loss_g.backward()
    loss_c.backward()
    gc = pm_c.head.lm_head.weight.grad
    gg = pm_g.head.lm_head.weight.grad.cpu()
    assert (gc - gg).abs().max() < 5e-2 * gc.abs().max()


def test_embedding_row_flags_equal_zeroed_gradient_bitwise(monkeypatch):
    """Skipping the embedding rows a step did not touch (flags from the sorted embedding
    backward, read as gradient 0 by the norm and AdamW kernels) gives bit-identical
    training to zeroing the whole embedding gradient every step."""
    cfg = _cfg()
    corpus = _corpus(cfg)
    monkeypatch.setenv("ODP_FUSED_NORM", "0")  # the same gradient-norm pass in both runs
    monkeypatch.setenv("ODP_EMB_ROWS", "1")
    a = _engine(cfg, "cuda")
    ha = a.fit(corpus, 3, 4, log_every=0)
    assert a._fused.emb_rows is not None
    monkeypatch.setenv("ODP_EMB_ROWS", "0")
    b = _engine(cfg, "cuda")
    hb = b.fit(corpus, 3, 4, log_every=0)
    assert b._fused.emb_rows is None
    assert [m.per_path_loss for m in ha] == [m.per_path_loss for m in hb]
    assert _bank_maxdiff(a, b) == 0.0


def test_fused_gradient_norm_matches_gradient_pass(monkeypatch):
    """The clip norm assembled from the producers' sums of squares (GEMM epilogue boxes,
    embedding rows, norm weights) equals the norm of a separate pass over the gradients
    (summation order differs: fp32 rounding only)."""
    cfg = _cfg()
    corpus = _corpus(cfg)
    runs = {}
    for flag in ("1", "0"):
        monkeypatch.setenv("ODP_FUSED_NORM", flag)
        eng = _engine(cfg, "cuda")
        eng.fit(corpus, 2, 4, log_every=0)
        assert (eng._fused.sq_bases is not None) == (flag == "1")
        runs[flag] = (eng._fused.GNORM.clone(), eng)
    a, b = runs["1"][0], runs["0"][0]
    assert torch.all(a > 0)
    assert torch.allclose(a, b, rtol=2e-5, atol=0), (a, b)
    assert _bank_maxdiff(runs["1"][1], runs["0"][1]) < 1e-4


def test_lookahead_fit_equals_round_by_round_bitwise():
    """fit(num_rounds=3) samples each next round's batches while the GPU runs the current
    one; training is bit-identical to three fit(num_rounds=1) calls (same generator order)."""
    cfg = _cfg()
    corpus = _corpus(cfg)
    a, b = _engine(cfg, "cuda"), _engine(cfg, "cuda")
    a.total_rounds = b.total_rounds = 3
    ha = a.fit(corpus, 3, 4, log_every=0)
    hb = [m for _ in range(3) for m in b.fit(corpus, 1, 4, log_every=0)]
    assert [m.per_path_loss for m in ha] == [m.per_path_loss for m in hb]
    assert _bank_maxdiff(a, b) == 0.0
    assert torch.equal(a._gen.get_state(), b._gen.get_state())


def test_split_k_weight_gradients_track_unsplit(monkeypatch):
    """Forcing the K split of every weight-gradient GEMM (fixed-order reduction of the
    splits) trains like the unsplit GEMMs up to fp32 summation order."""
    cfg = _cfg()
    corpus = _corpus(cfg)
    runs = {}
    for forced in ("2", "1"):
        monkeypatch.setenv("ODP_SPLITK", forced)
        eng = _engine(cfg, "cuda")
        h = eng.fit(corpus, 2, 4, log_every=0)
        assert max(eng._fused.wg_split.values()) == int(forced)
        runs[forced] = (h, eng)
    for a, b in zip(runs["2"][0], runs["1"][0]):
        for p in a.per_path_loss:
            assert abs(a.per_path_loss[p] - b.per_path_loss[p]) < 1e-3 * b.per_path_loss[p]
    assert _bank_maxdiff(runs["2"][1], runs["1"][1]) < 1e-3


def _bank_equal(a, b):
    for k in a.bank:
        for x, y in zip(a.bank[k].state_dict().values(), b.bank[k].state_dict().values()):
            if not torch.equal(x, y):
                return False
    return True


def test_activation_checkpoint_recompute_is_bitwise():
    """Checkpointing keeps only the layer inputs and recomputes each layer's forward
    before its backward with the same deterministic kernels: identical training."""
    cfg = _cfg(layers=(2, 1))
    corpus = _corpus(cfg)
    a, b = _engine(cfg, "cuda"), _engine(cfg, "cuda", activation_checkpoint=True)
    ha, hb = a.fit(corpus, 3, 4, log_every=0), b.fit(corpus, 3, 4, log_every=0)
    assert b._fused.ckpt and b._fused.QKV.shape[0] == 1 and a._fused.QKV.shape[0] == 3
    assert [m.per_path_loss for m in ha] == [m.per_path_loss for m in hb]
    assert _bank_equal(a, b)


@pytest.mark.parametrize("vocab_impl", ["fused", "partials"])
def test_loss_chunks_track_the_whole_batch(vocab_impl, monkeypatch):
    """loss_chunks = 3 on a 6-sequence batch: the logits buffer holds 2 sequences, the
    loss is normalised by the whole batch, and training matches the unchunked run up to
    the weight-gradient summation order (exactly for the loss of the first step)."""
    if vocab_impl == "partials":
        monkeypatch.setenv("ODP_CE_IMPL", "partials")
    cfg = _cfg()
    corpus = _corpus(cfg)
    a, b = _engine(cfg, "cuda"), _engine(cfg, "cuda", loss_chunks=3)
    ha, hb = a.fit(corpus, 3, 6, log_every=0), b.fit(corpus, 3, 6, log_every=0)
    assert len(b._fused.chunks) == 3 and b._fused.LOGITS.shape[1] == 2 * 64
    for x, y in zip(ha, hb):
        for p in x.per_path_loss:
            assert abs(x.per_path_loss[p] - y.per_path_loss[p]) < 1e-3 * x.per_path_loss[p], (p, x, y)
    assert _bank_maxdiff(a, b) < 2e-3


@pytest.mark.parametrize("chunks", [1, 2])
def test_ce_gradient_gemms_train_bitwise_like_the_in_place_pass(chunks, monkeypatch):
    """Hidden 256: the LM-head gradient GEMMs form the dlogits themselves (the logits are
    read once by a stats-only CE pass and never rewritten); training is bit for bit the
    run with the in-place CE pass, unchunked and with two loss chunks."""
    bb = BackboneConfig(vocab_size=512, hidden_size=256, num_attention_heads=4, intermediate_size=512,
                        layers_per_level=[1, 1], max_position_embeddings=128)
    cfg = DiPaCoConfig(backbone=bb, level_sizes=[2, 2], sequence_length=64)
    corpus = _corpus(cfg)
    monkeypatch.setenv("ODP_CE_GRAD_FUSED", "1")
    a = _engine(cfg, "cuda", loss_chunks=chunks)
    ha = a.fit(corpus, 2, 8, log_every=0)
    assert a._fused.ce_xf
    monkeypatch.setenv("ODP_CE_GRAD_FUSED", "0")
    b = _engine(cfg, "cuda", loss_chunks=chunks)
    hb = b.fit(corpus, 2, 8, log_every=0)
    assert not b._fused.ce_xf
    assert [m.per_path_loss for m in ha] == [m.per_path_loss for m in hb]
    assert _bank_equal(a, b)
