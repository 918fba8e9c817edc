"""Numerics of the sm_100a kernels against plain PyTorch fp32 references."""

import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _bf(*shape, scale=1.0, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(DEV).to(torch.bfloat16)


def _close(a, b, tol):
    a, b = a.float(), b.float()
    err = (a - b).abs().max().item()
    ref = b.abs().max().item() + 1e-6
    assert err <= tol * ref, f"max err {err} vs ref max {ref} (tol {tol})"


def _check_err():
    from opendipaco_b200.ops import check_errors

    torch.cuda.synchronize()
    check_errors()


@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (256, 384, 384), (3072, 1152, 384), (200, 96, 136),
                                   (512, 256, 1024)])
@pytest.mark.parametrize("bn", [64, 128])
def test_gemm_nt(M, N, K, bn):
    from opendipaco_b200.ops.gemm import mm_nt

    a, b = _bf(M, K, seed=1), _bf(N, K, seed=2)
    c = mm_nt(a, b, bn=bn)
    _check_err()
    _close(c, a.float() @ b.float().T, 1e-2)


@pytest.mark.parametrize("M,N,K", [(256, 384, 384), (384, 1024, 256), (128, 64, 512)])
def test_gemm_nn_mn_major_b(M, N, K):
    from opendipaco_b200.ops.gemm import mm_nn

    a, b = _bf(M, K, seed=3), _bf(K, N, seed=4)
    c = mm_nn(a, b, out_dtype=torch.float32)
    _check_err()
    _close(c, a.float() @ b.float(), 2e-3)


@pytest.mark.parametrize("M,N,K", [(384, 384, 512), (1152, 384, 3072), (128, 128, 128)])
def test_gemm_tn_weight_grad(M, N, K):
    from opendipaco_b200.ops.gemm import mm_tn

    a, b = _bf(K, M, seed=5), _bf(K, N, seed=6)
    c = mm_tn(a, b)
    _check_err()
    _close(c, a.float().T @ b.float(), 2e-3)


def test_gemm_tt():
    from opendipaco_b200.ops.gemm import mm_tt

    a, b = _bf(256, 384, seed=7), _bf(128, 256, seed=8)
    c = mm_tt(a, b)
    _check_err()
    _close(c, a.float().T @ b.float().T, 2e-3)


def test_gemm_grouped_and_residual():
    from opendipaco_b200.ops.gemm import gemm

    G, M, N, K = 3, 256, 384, 384
    a, b = _bf(G, M, K, seed=9), _bf(G, N, K, seed=10)
    r = torch.randn(G, M, N, device=DEV)
    c = torch.empty(G, M, N, device=DEV)
    gemm(a, K, M * K, False, b, K, N * K, False, c, N, M * N, M, N, K, G=G, epi="resid", R=r, ldr=N, sr=M * N)
    _check_err()
    _close(c, r + torch.bmm(a.float(), b.float().transpose(1, 2)), 2e-3)


def test_gemm_swiglu_fwd_bwd():
    from opendipaco_b200.ops.gemm import gemm

    M, H, Fd = 256, 384, 1024
    x = _bf(M, H, seed=11)
    w = _bf(2 * Fd, H, scale=0.05, seed=12)  # [gate; up]
    h = torch.empty(M, Fd, device=DEV, dtype=torch.bfloat16)
    gu = torch.empty(M, 2 * Fd, device=DEV, dtype=torch.bfloat16)
    gemm(x, H, 0, False, w, H, 0, False, h, Fd, 0, M, 2 * Fd, H, epi="swiglu", bn=128, aux=gu, ldx=2 * Fd,
         f_half=Fd)
    _check_err()
    ref_gu = (x.float() @ w.float().T).to(torch.bfloat16)
    _close(gu, ref_gu, 1e-2)
    g, u = ref_gu[:, :Fd].float(), ref_gu[:, Fd:].float()
    ref_h = (F.silu(g).to(torch.bfloat16).float() * u)
    _close(h, ref_h, 2e-2)
    # backward: dH = dY Wd with Wd [H, F] (MN-major B); epilogue -> [dG | dU]
    dy = _bf(M, H, seed=13)
    wd = _bf(H, Fd, scale=0.05, seed=14)
    dgu = torch.empty(M, 2 * Fd, device=DEV, dtype=torch.bfloat16)
    gemm(dy, H, 0, False, wd, Fd, 0, True, dgu, 2 * Fd, 0, M, Fd, H, epi="swiglu_bwd", bn=128, aux=gu,
         ldx=2 * Fd, f_half=Fd)
    _check_err()
    dh = (dy.float() @ wd.float()).to(torch.bfloat16).float()
    gg, uu = gu[:, :Fd].float(), gu[:, Fd:].float()
    sg = torch.sigmoid(gg)
    du = dh * (gg * sg)
    dg = (dh * uu) * sg * (1 + gg * (1 - sg))
    _close(dgu[:, Fd:], du, 2e-2)
    _close(dgu[:, :Fd], dg, 2e-2)


def test_logits_and_cross_entropy():
    from opendipaco_b200.ops._ext import ext
    from opendipaco_b200.ops.gemm import gemm

    M, H, V = 384, 384, 32000
    x = _bf(M, H, seed=15)
    w = _bf(V, H, scale=0.05, seed=16)
    T = 2 * (V // 128)
    logits = torch.empty(M, V, device=DEV, dtype=torch.bfloat16)
    part = torch.empty(M, T, 2, device=DEV)
    gemm(x, H, 0, False, w, H, 0, False, logits, V, 0, M, V, H, epi="logits", bn=128, part=part)
    _check_err()
    ref = (x.float() @ w.float().T).to(torch.bfloat16)
    _close(logits, ref, 1e-2)
    labels = torch.randint(0, V, (M,), device=DEV, dtype=torch.int32)
    labels[5] = -100
    lse = torch.empty(M, device=DEV)
    rl = torch.empty(M, device=DEV)
    ls, ic, lo = torch.empty(1, device=DEV), torch.empty(1, device=DEV), torch.empty(1, device=DEV)
    ext().ce_forward(part, T, logits, V, 0, labels, M, 1, lse, rl, ls, ic, lo, None)
    lf = logits.float().requires_grad_(True)
    ref_loss = F.cross_entropy(lf, labels.long(), ignore_index=-100)
    ref_loss.backward()
    torch.cuda.synchronize()
    assert abs(lo.item() - ref_loss.item()) < 1e-3 * max(1.0, ref_loss.item())
    ext().ce_backward(logits, V, 0, lse, labels, ic, M, V, 1)
    _check_err()
    _close(logits, lf.grad, 2e-2)


@pytest.mark.parametrize("H", [384, 128, 512, 1024, 640])   # 640: no register-resident variant
def test_rmsnorm_fwd_bwd(H):
    from opendipaco_b200.ops.norm import rms_norm_bwd, rms_norm_fwd

    R = 300
    x = torch.randn(R, H, device=DEV)
    w = torch.rand(H, device=DEV) + 0.5
    y, rstd = rms_norm_fwd(x, w, 1e-5)
    xr = x.clone().requires_grad_(True)
    wr = w.clone().requires_grad_(True)
    yr = wr * (xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-5))
    _close(y, yr, 1e-2)
    dy = torch.randn(R, H, device=DEV)
    yr.backward(dy)
    dres = torch.randn(R, H, device=DEV)
    dx, dw = rms_norm_bwd(x, w, rstd, dy, dres)
    _check_err()
    _close(dx, xr.grad + dres, 1e-4)
    _close(dw, wr.grad, 1e-4)


@pytest.mark.parametrize("H", [128, 256, 384, 512, 1024])
def test_rmsnorm_fwd_four_rows_per_warp(H):
    """The 4-rows-per-warp forward (the production variant at 16 paths per GPU) on a row
    count that is not a multiple of 4, against the fp32 reference and against the
    one-row-per-warp launch of the same register width."""
    from opendipaco_b200.ops._ext import ext

    G, M = 2, 4737                      # G * M / 32 >= 2 * 148: the automatic choice is 4 rows per warp
    torch.manual_seed(H)
    x = torch.randn(G, M, H, device=DEV)
    w = torch.rand(G, H, device=DEV) + 0.5
    outs = {}
    for rpw in (0, 4, 1):
        y = torch.full((G, M, H), float("nan"), device=DEV, dtype=torch.bfloat16)
        rstd = torch.full((G, M), float("nan"), device=DEV)
        ext().rmsnorm_fwd_rpw(x, M * H, w, H, y, M * H, rstd, M, H, G, 1e-5, rpw)
        outs[rpw] = (y, rstd)
    torch.cuda.synchronize()
    rs_ref = torch.rsqrt(x.pow(2).mean(-1) + 1e-5)
    y_ref = w[:, None, :] * (x * rs_ref[..., None])
    for rpw, (y, rstd) in outs.items():
        assert not torch.isnan(y.float()).any() and not torch.isnan(rstd).any(), rpw
        _close(rstd, rs_ref, 1e-5)
        _close(y, y_ref, 1e-2)
    assert torch.equal(outs[0][0], outs[4][0]) and torch.equal(outs[0][1], outs[4][1])
    torch.testing.assert_close(outs[4][1], outs[1][1], rtol=1e-6, atol=0)
    torch.testing.assert_close(outs[4][0].float(), outs[1][0].float(), rtol=8e-3, atol=0)


def test_embedding_fwd_bwd_deterministic():
    from opendipaco_b200.ops.norm import embedding_bwd, embedding_fwd

    V, H = 1000, 384
    E = torch.randn(V, H, device=DEV)
    ids = torch.randint(0, 50, (4, 96), device=DEV)
    out = embedding_fwd(ids, E)
    _close(out, E[ids], 0)
    dx = torch.randn(4, 96, H, device=DEV)
    dE = embedding_bwd(ids, dx, V)
    ref = torch.zeros(V, H, device=DEV).index_add_(0, ids.reshape(-1), dx.reshape(-1, H))
    _close(dE, ref, 1e-5)
    assert torch.equal(dE, embedding_bwd(ids, dx, V))


def _rope_ref(x, cos, sin):
    h = x.shape[-1] // 2
    rot = torch.cat([-x[..., h:], x[..., :h]], -1)
    return x * cos + rot * sin


@pytest.mark.parametrize("B,S,nh,nkv", [(2, 128, 6, 6), (1, 256, 4, 2), (3, 64, 2, 1)])
def test_attention_fwd_bwd(B, S, nh, nkv):
    from opendipaco_b200.models.llama import rope_cos_sin
    from opendipaco_b200.ops.attention import attention_bwd, attention_fwd

    D = 64
    cos, sin = rope_cos_sin(D, 10000.0, S, DEV)
    qkv = _bf(B, S, (nh + 2 * nkv) * D, seed=17)
    o, lse = attention_fwd(qkv, nh, nkv, cos, sin)
    _check_err()
    x = qkv.float().requires_grad_(True)
    q = x[..., :nh * D].view(B, S, nh, D).transpose(1, 2)
    k = x[..., nh * D:(nh + nkv) * D].view(B, S, nkv, D).transpose(1, 2)
    v = x[..., (nh + nkv) * D:].view(B, S, nkv, D).transpose(1, 2)
    q, k = _rope_ref(q, cos, sin), _rope_ref(k, cos, sin)
    rep = nh // nkv
    k, v = k.repeat_interleave(rep, 1), v.repeat_interleave(rep, 1)
    ref = F.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(1, 2).reshape(B, S, nh * D)
    _close(o, ref, 2e-2)
    do = _bf(B, S, nh * D, seed=18)
    ref.backward(do.float())
    dqkv = attention_bwd(qkv, o, lse, do, nh, nkv, cos, sin)
    _check_err()
    _close(dqkv, x.grad, 3e-2)


def test_adamw_matches_torch():
    from opendipaco_b200.ops.adam import adamw, clip_coef, sched_tensor

    G, P = 2, 4096 * 3
    p = torch.randn(G, P, device=DEV)
    g = torch.randn(G, P, device=DEV)
    m, v = torch.zeros_like(p), torch.zeros_like(p)
    p16 = torch.empty(G, P, device=DEV, dtype=torch.bfloat16)
    ref = [torch.nn.Parameter(p[i].clone()) for i in range(G)]
    opts = [torch.optim.AdamW([r], lr=1e-3, betas=(0.9, 0.95), weight_decay=0.1) for r in ref]
    for step in range(1, 4):
        for i in range(G):
            ref[i].grad = g[i].clone()
            torch.nn.utils.clip_grad_norm_([ref[i]], 1.0)
            opts[i].step()
        coef = clip_coef(g, P, P, G, 1.0)
        adamw(p, g, m, v, p16, P, P, P, G, coef, sched_tensor(1e-3, 0.9, 0.95, step, DEV, groups=G), 0.9, 0.95, 1e-8, 0.1)
    _check_err()
    for i in range(G):
        _close(p[i], ref[i].detach(), 1e-5)
    _close(p16, p, 1e-2)


def test_adam8bit_cuda_matches_cpu():
    from opendipaco_b200.optim.adam8bit import Adam8bit

    torch.manual_seed(0)
    w = torch.randn(1000, 3)
    pc = torch.nn.Parameter(w.clone())
    pg = torch.nn.Parameter(w.clone().to(DEV))
    oc = Adam8bit([pc], lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1)
    og = Adam8bit([pg], lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1)
    for _ in range(5):
        gr = torch.randn(1000, 3)
        pc.grad, pg.grad = gr.clone(), gr.clone().to(DEV)
        oc.step()
        og.step()
    _check_err()
    _close(pg.detach().cpu(), pc.detach(), 1e-4)
    sc, sg = oc.state[pc], og.state[pg]
    assert (sc["m_q"].int() - sg["m_q"].cpu().int()).abs().max() <= 1


def test_outer_step_matches_torch_sgd():
    from opendipaco_b200.ops.outer import OuterPlan, Segment

    n = 10000
    glob = torch.randn(n, device=DEV)
    mom = torch.zeros(n, device=DEV)
    locs = [glob + 0.01 * torch.randn(n, device=DEV) for _ in range(3)]
    l16 = [torch.empty(n, device=DEV, dtype=torch.bfloat16) for _ in range(3)]
    w = [0.2, 0.3, 0.5]
    p = torch.nn.Parameter(glob.clone())
    sgd = torch.optim.SGD([p], lr=0.7, momentum=0.9, nesterov=True)
    plan = OuterPlan([Segment("k", glob, mom, locs, l16, w, scale=math.sqrt(3))], DEV)
    for it in range(3):
        acc = torch.zeros(n, device=DEV)
        for wi, l in zip(w, locs):
            acc.add_(wi * (p.detach() - l))
        p.grad = acc * math.sqrt(3)
        sgd.step()
        plan.run(0.7, 0.9, True, first=(it == 0))
        torch.cuda.synchronize()
        _close(glob, p.detach(), 1e-6)
        for l in locs:
            assert torch.equal(l, glob)
            l.add_(0.01 * torch.randn(n, device=DEV))
        p.data.copy_(glob)


def test_peer_copy_segments_with_tails():
    """The pull-copy kernel (used over NVLink for the full-bank gather) on local memory:
    many segments, lengths not multiples of 4, one launch."""
    from opendipaco_b200.ops._ext import ext

    g = torch.Generator().manual_seed(3)
    srcs = [torch.randn(n, generator=g).cuda() for n in (1, 4, 7, 1000, 4099, 70001)]
    dsts = [torch.zeros_like(s) for s in srcs]
    tab = torch.tensor([[s.data_ptr(), d.data_ptr(), s.numel()] for s, d in zip(srcs, dsts)],
                       dtype=torch.int64).cuda()
    ext().peer_copy(tab, max(s.numel() for s in srcs))
    torch.cuda.synchronize()
    for s, d in zip(srcs, dsts):
        assert torch.equal(s, d)
