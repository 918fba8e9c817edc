"""Warm start from a pretrained dense Llama (models/init.py): layers copied by depth, the
warm-started path reproduces the pretrained logits, and the discriminative router
(routing/discriminative.py), both against the reference's results."""

import torch

from opendipaco_b200 import BackboneConfig, DiPaCoConfig
from opendipaco_b200.models.init import warm_start_modules
from opendipaco_b200.models.path import build_module_bank
from opendipaco_b200.routing.discriminative import DiscriminativeRouter


def _hf_llama(bb: BackboneConfig, layers: int):
    from transformers import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig(vocab_size=bb.vocab_size, hidden_size=bb.hidden_size, intermediate_size=bb.intermediate_size,
                      num_hidden_layers=layers, num_attention_heads=bb.num_attention_heads,
                      num_key_value_heads=bb.kv_heads(), max_position_embeddings=bb.max_position_embeddings,
                      tie_word_embeddings=False)
    torch.manual_seed(5)
    return LlamaForCausalLM(cfg).eval()


def test_warm_start_copies_pretrained_layers_by_depth():
    bb = BackboneConfig(vocab_size=300, hidden_size=64, num_attention_heads=4, intermediate_size=128,
                        layers_per_level=[1, 2], max_position_embeddings=64)
    cfg = DiPaCoConfig(backbone=bb, level_sizes=[2, 2], sequence_length=32)
    topo = cfg.build_topology()
    bank = build_module_bank(cfg, seed=0)
    hf = _hf_llama(bb, 4)
    warm_start_modules(bank, topo, hf)
    sd = hf.state_dict()
    assert torch.equal(bank["embed"].embed_tokens.weight, sd["model.embed_tokens.weight"])
    assert torch.equal(bank["head"].lm_head.weight, sd["lm_head.weight"])
    assert torch.equal(bank["head"].norm.weight, sd["model.norm.weight"])
    for key, mod in bank.items():
        if topo.role_of_key(key) in ("embed", "head"):
            continue
        off = topo.offset_of_key(key)
        for j, layer in enumerate(mod.layers):
            for name, p in layer.named_parameters():
                assert torch.equal(p, sd[f"model.layers.{off + j}.{name}"]), (key, j, name)


def test_warm_start_matches_reference(reference_pkg):
    from opendipaco import BackboneConfig as RB, DiPaCoConfig as RC
    from opendipaco.init import warm_start_modules as ref_warm
    from opendipaco.model import build_module_bank as ref_bank

    kw = dict(vocab_size=300, hidden_size=64, num_attention_heads=4, intermediate_size=128,
              layers_per_level=[2, 1], max_position_embeddings=64)
    cfg = DiPaCoConfig(backbone=BackboneConfig(**kw), level_sizes=[2, 1], sequence_length=32)
    rcfg = RC(backbone=RB(**kw), level_sizes=[2, 1], sequence_length=32)
    hf = _hf_llama(BackboneConfig(**kw), 3)
    ours, theirs = build_module_bank(cfg, seed=1), ref_bank(rcfg, seed=1)
    warm_start_modules(ours, cfg.build_topology(), hf)
    ref_warm(theirs, rcfg.build_topology(), hf)
    for key in theirs:
        a, b = ours[key].state_dict(), theirs[key].state_dict()
        for n in b:
            assert torch.equal(a[n], b[n]), (key, n)


def test_discriminative_router_matches_reference(reference_pkg):
    from opendipaco.routing.discriminative import DiscriminativeRouter as Ref

    g = torch.Generator().manual_seed(0)
    x = torch.randn(200, 16, generator=g)
    y = (x[:, 0] > 0).long() + 2 * (x[:, 1] > 0).long()
    for val in (0.0, 0.25):
        torch.manual_seed(3)
        ours = DiscriminativeRouter(16, 4).fit(x, y, epochs=60, val_fraction=val, seed=1)
        torch.manual_seed(3)
        theirs = Ref(16, 4).fit(x, y, epochs=60, val_fraction=val, seed=1)
        for n, t in theirs.state_dict().items():
            assert torch.equal(ours.state_dict()[n], t)
        assert (ours.predict(x) == y).float().mean() > 0.75
        assert ours.predict_topk(x, 9).shape == (200, 4)


def test_warm_started_path_reproduces_the_pretrained_logits():
    """A path whose modules were warm-started from a pretrained Llama of the same depth
    computes that model's logits (fp32, same token ids)."""
    from opendipaco_b200.models.path import build_path_model

    bb = BackboneConfig(vocab_size=300, hidden_size=64, num_attention_heads=4, num_key_value_heads=2,
                        intermediate_size=128, layers_per_level=[1, 2], max_position_embeddings=64)
    cfg = DiPaCoConfig(backbone=bb, level_sizes=[2, 2], sequence_length=32)
    topo = cfg.build_topology()
    bank = build_module_bank(cfg, seed=0)
    hf = _hf_llama(bb, 3)
    hf.config.rms_norm_eps = bb.rms_norm_eps  # the pretrained model's norm epsilon matches the backbone's
    for m in hf.modules():
        if hasattr(m, "variance_epsilon"):
            m.variance_epsilon = bb.rms_norm_eps
    warm_start_modules(bank, topo, hf)
    ids = torch.randint(0, 300, (2, 24), generator=torch.Generator().manual_seed(0))
    with torch.no_grad():
        want = hf(input_ids=ids).logits
        for p in range(cfg.num_paths):
            model = build_path_model(cfg, topo.path_from_index(p), bank).eval()
            out = model(ids)
            got = out[0] if isinstance(out, tuple) else out
            torch.testing.assert_close(got, want, rtol=1e-4, atol=1e-4)


def test_eval_sequence_length_defaults_and_validation():
    import pytest

    bb = BackboneConfig(vocab_size=64, hidden_size=32, num_attention_heads=4, intermediate_size=64,
                        layers_per_level=[1, 1], max_position_embeddings=256)
    assert DiPaCoConfig(backbone=bb, level_sizes=[2, 2], sequence_length=32).eval_seq_len == 32
    assert DiPaCoConfig(backbone=bb, level_sizes=[2, 2], sequence_length=32,
                        eval_sequence_length=128).eval_seq_len == 128
    with pytest.raises(ValueError):
        DiPaCoConfig(backbone=bb, level_sizes=[2, 2], sequence_length=32, eval_sequence_length=0)
