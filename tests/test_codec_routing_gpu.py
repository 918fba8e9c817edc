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


def _ref_sqd(x, c):
    x64, c64 = x.double(), c.double()
    return (x64 * x64).sum(1, keepdim=True) - 2 * x64 @ c64.T + (c64 * c64).sum(1)


@pytest.mark.parametrize("N,K,D,k", [(300, 8, 64, 3), (1000, 16, 256, 1), (777, 20, 40, 4),
                                     (513, 300, 96, 8), (129, 256, 256, 2)])
def test_tensor_core_assignment_matches_fp64(N, K, D, k):
    """The tcgen05 3xTF32 distances match an fp64 reference to fp32 accuracy and the k
    nearest agree wherever the distance gap is resolvable (K > 256: several blocks; K and
    D not multiples of 16 / 32: padded columns)."""
    from opendipaco_b200.ops import routing as R

    g = torch.Generator().manual_seed(N + K)
    x = torch.randn(N, D, generator=g)
    c = torch.randn(K, D, generator=g)
    idx, mind, dist = R.assign(x.cuda(), c.cuda(), k, want_min=True, want_dist=True)
    ref = _ref_sqd(x, c)
    scale = (x.norm(dim=1, keepdim=True) * c.norm(dim=1)).double()
    assert ((dist.cpu().double() - ref).abs() <= 2e-6 * scale + 1e-5).all()
    srt, order = ref.sort(dim=1, stable=True)
    idx = idx.cpu()
    for j in range(k):
        gap = torch.minimum(srt[:, j + 1] - srt[:, j] if j + 1 < K else torch.full((N,), 1e9, dtype=torch.float64),
                            srt[:, j] - srt[:, j - 1] if j > 0 else torch.full((N,), 1e9, dtype=torch.float64))
        clear = gap > 1e-3 * scale.max(dim=1).values
        assert torch.equal(idx[clear, j], order[clear, j])
    assert ((mind.cpu().double() - srt[:, 0]).abs() <= 2e-6 * scale.max(dim=1).values + 1e-5).all()
    from opendipaco_b200.ops._ext import check_errors

    check_errors()


def test_cluster_sums_deterministic_and_exact():
    from opendipaco_b200.ops import routing as R

    g = torch.Generator().manual_seed(7)
    N, K, D = 5000, 13, 200
    x = torch.randn(N, D, generator=g).cuda()
    a = torch.randint(0, K, (N, 2), generator=g).cuda()
    a[:, 0][a[:, 0] == 5] = 6  # cluster 5 stays empty
    s1, n1 = R.cluster_sums(x, a, K)
    s2, n2 = R.cluster_sums(x, a, K)
    assert torch.equal(s1, s2) and torch.equal(n1, n2)
    ref = torch.zeros(K, D, dtype=torch.float64).index_add_(0, a[:, 0].cpu(), x.cpu().double())
    assert torch.allclose(s1.cpu().double(), ref, atol=1e-3)
    assert torch.equal(n1.cpu().long(), torch.bincount(a[:, 0].cpu(), minlength=K))
    assert int(n1[5]) == 0 and float(s1[5].abs().sum()) == 0.0


def test_device_kmeans_fit_matches_cpu_fit():
    """Well separated blobs: the device fit (tensor-core assignment, ordered sums) finds
    the same clusters as the reference-style CPU loop, and is reproducible bit for bit."""
    from opendipaco_b200.routing import KMeansRouter

    g = torch.Generator().manual_seed(11)
    centers = torch.randn(6, 64, generator=g) * 10
    pts = torch.cat([centers[i] + torch.randn(400, 64, generator=g) for i in range(6)])
    rc = KMeansRouter(6, seed=0).fit(pts)
    # the same initial centroids as the CPU fit (randperm differs between devices)
    cent0 = pts[torch.randperm(len(pts), generator=torch.Generator().manual_seed(0))[:6]]
    r = KMeansRouter(6, seed=0)
    c1 = r._fit_device(pts.cuda(), cent0.cuda())
    c2 = r._fit_device(pts.cuda(), cent0.cuda())
    assert torch.equal(c1, c2)
    assert torch.allclose(rc.centroids, c1.cpu(), atol=1e-4)
    r.centroids = c1
    assert torch.equal(rc.predict(pts), r.predict(pts.cuda()).cpu())
    assert KMeansRouter(6, seed=0).fit(pts.cuda()).centroids.shape == (6, 64)
