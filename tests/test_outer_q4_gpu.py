"""Compressed NVLink outer step (csrc/outer_nvlink.cu). int4: the QUANT kernel against an
fp32 PyTorch restatement of group-128 absmax/7 quantisation with error feedback, and the
compressed APPLY path (one GPU, one sharer) against dequantise + Nesterov in PyTorch.
top-k: the TOPK kernel against a sort-based per-block top-k (ties in index order) and
the pair-summing APPLY path against Nesterov on the kept entries."""

import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"
G = 128


def _ref_quant(x):
    g = x.view(-1, G)
    am = g.abs().amax(1)
    sc = am / torch.full_like(am, 7.0)   # a true division (a scalar divisor becomes a reciprocal multiply)
    safe = torch.where(sc > 0, sc, torch.ones_like(sc))
    q = torch.clamp(torch.round(g / safe[:, None]), -7, 7)
    res = g - q * sc[:, None]
    return q.view(-1), sc, res.view(-1)


def _unpack(qd_bytes):
    b = qd_bytes.to(torch.int32)
    return torch.stack([(b & 15) - 8, (b >> 4) - 8], 1).view(-1)


def _regions(spans):
    from opendipaco_b200.parallel.backend.nvlink import NVREGION

    arr, g0 = np.zeros(len(spans), dtype=NVREGION), 0
    for i, (off, n) in enumerate(spans):
        arr[i] = (off, n, g0)
        g0 += n // G
    return torch.from_numpy(arr.view(np.int64).copy()).to(DEV), len(spans), g0


def test_quant_kernel_matches_reference_with_error_feedback():
    from opendipaco_b200.ops._ext import ext

    gen = torch.Generator(device="cpu").manual_seed(0)
    total = 4096
    delta = torch.randn(total, generator=gen).to(DEV) * torch.logspace(-3, 1, total // G).repeat_interleave(G).to(DEV)
    delta[1024:1152] = 0.0                       # an all-zero group: scale 0, codes 0
    res = torch.randn(total, generator=gen).to(DEV) * 1e-3
    spans = [(0, 1536), (2048, 1024), (3584, 256)]   # regions in key order; the gaps stay untouched
    regs, nregs, groups = _regions(spans)
    qd = torch.full((total // 2,), 0xAA, dtype=torch.uint8, device=DEV)
    qs = torch.full((total // G,), -1.0, device=DEV)
    res_k = res.clone()
    ext().outer_nvlink_quant(regs, nregs, groups, delta, res_k, qd, qs)
    torch.cuda.synchronize()
    for off, n in spans:
        q, sc, r = _ref_quant(delta[off:off + n] + res[off:off + n])
        assert torch.equal(_unpack(qd[off // 2:(off + n) // 2]), q.to(torch.int32))
        assert torch.equal(qs[off // G:(off + n) // G], sc)
        assert torch.equal(res_k[off:off + n], r)
    assert torch.all(qd[1536 // 2:2048 // 2] == 0xAA) and torch.all(qs[1536 // G:2048 // G] == -1.0)
    assert torch.equal(res_k[1536:2048], res[1536:2048])
    # error feedback: what the first outer step dropped is carried into the second step's codes
    q1 = _unpack(qd[:768]).float() * qs[:12].repeat_interleave(G)
    ext().outer_nvlink_quant(regs, nregs, groups, delta, res_k, qd, qs)
    torch.cuda.synchronize()
    q2 = _unpack(qd[:768]).float() * qs[:12].repeat_interleave(G)
    two = 2 * delta[:1536] + res[:1536]
    assert torch.allclose(q1 + q2 + res_k[:1536], two, atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("first,nesterov", [(True, True), (False, True), (False, False)])
def test_compressed_apply_one_sharer_matches_reference(first, nesterov):
    from opendipaco_b200.ops._ext import check_errors, err_word, ext
    from opendipaco_b200.parallel.backend.nvlink import NVKEY

    gen = torch.Generator(device="cpu").manual_seed(1)
    n, off = 3000, 256                       # key region at element 256, size not a multiple of 128
    total = 4096
    delta = torch.zeros(total, device=DEV)
    delta[off:off + n] = torch.randn(n, generator=gen).to(DEV)
    glob = torch.zeros(total, device=DEV)
    glob[off:off + n] = torch.randn(n, generator=gen).to(DEV)
    mom = torch.zeros(total, device=DEV)
    mom[off:off + n] = torch.randn(n, generator=gen).to(DEV) * 0.1
    res = torch.zeros(total, device=DEV)
    qd = torch.zeros(total // 2, dtype=torch.uint8, device=DEV)
    qs = torch.zeros(total // G, device=DEV)
    n_r = (n + G - 1) // G * G
    regs, nregs, groups = _regions([(off, n_r)])
    ext().outer_nvlink_quant(regs, nregs, groups, delta, res, qd, qs)
    deq = _unpack(qd).float() * qs.repeat_interleave(G)

    chunk = int(ext().outer_nvlink_chunk_elems())
    s1 = n
    rec = np.zeros(1, dtype=NVKEY)
    rec["off"], rec["s0"], rec["s1"], rec["chunk0"], rec["nsh"] = off, 0, s1, 0, 1
    rec["sh"][0, 0] = 0
    rec["scale"], rec["inv_den"], rec["quant"] = 0.5, 0.25, 1
    keys = torch.from_numpy(rec.view(np.int64).copy()).to(DEV)
    nch = (s1 + chunk - 1) // chunk
    pad = torch.zeros(2, dtype=torch.int32, device=DEV)
    ptr = lambda t: torch.tensor([t.data_ptr()], dtype=torch.int64, device=DEV)  # noqa: E731
    sq = torch.zeros(nch, device=DEV)
    lr, m = 0.7, 0.9
    g0, m0 = glob.clone(), mom.clone()
    ext().outer_nvlink_apply(keys, 1, nch, ptr(delta), ptr(glob), ptr(pad), mom, 0, 1, 1, lr, m, nesterov, first,
                             sq, err_word(torch.device(DEV)), ptr(qd), ptr(qs), 0, None)
    torch.cuda.synchronize()
    check_errors()
    d = deq[off:off + n] * 0.25 * 0.5
    b = d if first else m0[off:off + n] * m + d
    upd = d + m * b if nesterov else b
    assert torch.allclose(mom[off:off + n], b, atol=1e-6, rtol=1e-6)
    assert torch.allclose(glob[off:off + n], g0[off:off + n] - lr * upd, atol=1e-5, rtol=1e-5)
    assert abs(sq.sum().item() - (d * d).sum().item()) <= 1e-3 * (d * d).sum().item()
    # int4 codes carry the partial to within half a quantisation step per element
    step = qs.repeat_interleave(G)[off:off + n]
    assert torch.all((deq[off:off + n] - delta[off:off + n]).abs() <= step / 2 + 1e-6)


def _ref_topk(x, density):
    """Per-4096-block top-k by magnitude (ties in index order) of a region of true size n."""
    out_idx, out_val, keep = [], [], torch.zeros_like(x, dtype=torch.bool)
    n = x.numel()
    for b0 in range(0, n, 4096):
        blk = x[b0:b0 + 4096]
        k = max(1, math.ceil(density * blk.numel()))
        # stable order: larger magnitude first, lower index first among equals
        mag = blk.abs().double()
        order = sorted(range(blk.numel()), key=lambda i: (-mag[i].item(), i))[:k]
        order.sort()
        keep[b0 + torch.tensor(order)] = True
        out_idx.append(torch.tensor(order, dtype=torch.int64))
        out_val.append(blk[torch.tensor(order)])
    return out_idx, out_val, keep


def test_topk_kernel_matches_reference_and_carries_the_rest():
    from opendipaco_b200.ops._ext import ext

    gen = torch.Generator(device="cpu").manual_seed(5)
    n, off, density = 9000, 4096, 0.01        # three blocks, the last one partial (808 elements)
    total = 4096 * 4
    kcap = math.ceil(density * 4096)
    delta = torch.zeros(total, device=DEV)
    delta[off:off + n] = torch.randn(n, generator=gen).to(DEV)
    res = torch.zeros(total, device=DEV)
    res[off:off + n] = torch.randn(n, generator=gen).to(DEV) * 0.01
    # 60 equal magnitudes at the top of block 1 (k = 41): the lowest indices win the tie
    delta[off + 4096 + 200:off + 4096 + 260] = 5.0
    delta[off + 4096 + 230:off + 4096 + 240] = -5.0
    res[off + 4096 + 200:off + 4096 + 260] = 0.0
    regs = torch.tensor([[off, n, 0]], dtype=torch.int64, device=DEV)
    spi = torch.zeros(total // 4096 * kcap, dtype=torch.int16, device=DEV)
    spv = torch.zeros(total // 4096 * kcap, device=DEV)
    x = (delta + res)[off:off + n].clone()
    res_k = res.clone()
    ext().outer_nvlink_topk(regs, 1, 3, density, kcap, delta, res_k, spi, spv)
    torch.cuda.synchronize()
    idx, val, keep = _ref_topk(x.cpu(), density)
    for b in range(3):
        slot = (off // 4096 + b) * kcap
        got_i = spi[slot:slot + kcap].to(torch.int64).cpu() & 0xFFFF
        got_v = spv[slot:slot + kcap].cpu()
        k = idx[b].numel()
        assert torch.equal(got_i[:k], idx[b]) and torch.equal(got_v[:k], val[b])
        assert torch.all(got_i[k:] == 0xFFFF) and torch.all(got_v[k:] == 0)
    r = res_k[off:off + n].cpu()
    assert torch.equal(r[keep], torch.zeros(int(keep.sum())))
    assert torch.equal(r[~keep], x.cpu()[~keep])
    assert torch.all(res_k[:off] == 0) and torch.all(res_k[off + n:] == 0)


def test_topk_apply_one_sharer_matches_reference():
    from opendipaco_b200.ops._ext import check_errors, err_word, ext
    from opendipaco_b200.parallel.backend.nvlink import NVKEY

    gen = torch.Generator(device="cpu").manual_seed(6)
    n, off, density = 6000, 4096, 0.05
    total = 4096 * 4
    kcap = math.ceil(density * 4096)
    delta = torch.zeros(total, device=DEV)
    delta[off:off + n] = torch.randn(n, generator=gen).to(DEV)
    glob = torch.zeros(total, device=DEV)
    glob[off:off + n] = torch.randn(n, generator=gen).to(DEV)
    mom = torch.zeros(total, device=DEV)
    res = torch.zeros(total, device=DEV)
    spi = torch.zeros(total // 4096 * kcap, dtype=torch.int16, device=DEV)
    spv = torch.zeros(total // 4096 * kcap, device=DEV)
    regs = torch.tensor([[off, n, 0]], dtype=torch.int64, device=DEV)
    ext().outer_nvlink_topk(regs, 1, 2, density, kcap, delta, res, spi, spv)
    sparse = delta - res                       # what the pairs carry
    rec = np.zeros(1, dtype=NVKEY)
    rec["off"], rec["s0"], rec["s1"], rec["chunk0"], rec["nsh"] = off, 0, n, 0, 1
    rec["sh"][0, 0] = 0
    rec["scale"], rec["inv_den"], rec["quant"] = 1.0, 1.0, 2
    keys = torch.from_numpy(rec.view(np.int64).copy()).to(DEV)
    pad = torch.zeros(2, dtype=torch.int32, device=DEV)
    ptr = lambda t: torch.tensor([t.data_ptr()], dtype=torch.int64, device=DEV)  # noqa: E731
    sq = torch.zeros(2, device=DEV)
    g0 = glob.clone()
    ext().outer_nvlink_apply(keys, 1, 2, ptr(delta), ptr(glob), ptr(pad), mom, 0, 1, 1, 0.7, 0.9, True, True, sq,
                             err_word(torch.device(DEV)), ptr(spi), ptr(spv), kcap, None)
    torch.cuda.synchronize()
    check_errors()
    d = sparse[off:off + n]
    assert int((d != 0).sum()) <= 2 * kcap
    assert torch.allclose(mom[off:off + n], d, atol=0, rtol=0)
    assert torch.allclose(glob[off:off + n], g0[off:off + n] - 0.7 * (d + 0.9 * d), atol=1e-6, rtol=1e-6)
