"""GPU codec / routing kernels against the PyTorch CPU implementations."""

import pytest
import torch

from opendipaco_b200.schedule import compress as C

pytestmark = pytest.mark.gpu


def test_int4_quant_matches_cpu_and_roundtrips():
    torch.manual_seed(0)
    x = torch.randn(1000, 33) * 0.01
    pc, rc = C._quantize_int4(x)
    pg, rg = C._quantize_int4(x.cuda())
    assert torch.equal(pc["q4"], pg["q4"].cpu()) and torch.allclose(pc["s"], pg["s"].cpu())
    assert torch.allclose(rc, rg.cpu(), atol=1e-7)
    d = C._dequant_int4({k: (v.cuda() if torch.is_tensor(v) else v) for k, v in pc.items()})
    assert torch.allclose(d.cpu(), C._dequant_int4(pc), atol=0)


def test_int8_quant_matches_cpu():
    torch.manual_seed(1)
    x = torch.randn(4096, 7)
    pc, rc = C._quantize_int8(x)
    pg, rg = C._quantize_int8(x.cuda())
    assert torch.equal(pc["q"], pg["q"]) and abs(pc["s"] - pg["s"]) < 1e-12
    assert torch.allclose(rc, rg.cpu(), atol=1e-7)


def test_decode_accumulate_fused():
    from opendipaco_b200.ops import codec

    torch.manual_seed(2)
    x = torch.randn(5000).cuda()
    packed, scale, _ = codec.quant_int4(x)
    acc = torch.ones(5000, device="cuda")
    codec.dequant_int4(packed, scale, 5000, out=acc, weight=0.5, accumulate=True)
    ref = 1 + 0.5 * codec.dequant_int4(packed, scale, 5000)
    assert torch.allclose(acc, ref)


@pytest.mark.parametrize("mode", ["mean", "trimmed_mean", "median"])
def test_robust_combine_matches_cpu(mode):
    from opendipaco_b200.schedule.aggregate import robust_delta

    torch.manual_seed(3)
    contribs = [(1.0, [torch.randn(300, 7)]) for _ in range(5)]
    dc, wc = robust_delta(contribs, aggregate=mode)
    dg, wg = robust_delta([(w, [g[0].cuda()]) for w, g in contribs], aggregate=mode)
    assert wc == wg and torch.allclose(dc[0], dg[0].cpu(), atol=1e-6)


def test_kmeans_assign_and_bag_of_tokens():
    from opendipaco_b200.routing import BagOfTokensFeaturizer, KMeansRouter

    torch.manual_seed(4)
    pre = [torch.randint(0, 5000, (32,)) for _ in range(300)]
    fc = BagOfTokensFeaturizer(5000, feature_dim=64)(pre)
    fg = BagOfTokensFeaturizer(5000, feature_dim=64, device="cuda")(pre)
    assert torch.allclose(fc, fg, atol=1e-6)
    r = KMeansRouter(8, seed=0).fit(fc)
    assert torch.equal(r.predict(fc), r.predict(fc.cuda()).cpu())
    assert torch.equal(r.predict_topk(fc, 3), r.predict_topk(fc.cuda(), 3).cpu())
