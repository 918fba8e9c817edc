"""CTA-pair (cta_group::2) GEMM against an fp32 PyTorch reference and against the
single-CTA kernel (ODP_GEMM_2SM=0), for every operand-major combination, grouped
problems, partial tiles (M not a multiple of 256) and the LM-head shapes."""

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _bf(*shape, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randn(*shape, generator=g).to(DEV).to(torch.bfloat16)


def _close(a, b, tol):
    a, b = a.float(), b.float()
    err = (a - b).abs().max().item()
    ref = b.abs().max().item() + 1e-6
    assert err <= tol * ref, f"max err {err} vs ref max {ref} (tol {tol})"


def _run(fn, monkeypatch, pair: bool):
    from opendipaco_b200.ops import check_errors

    monkeypatch.setenv("ODP_GEMM_2SM", "1" if pair else "0")
    out = fn()
    torch.cuda.synchronize()
    check_errors()
    return out


@pytest.mark.parametrize("G,M,N,K,a_mn,b_mn,epi", [
    (2, 3072, 32000, 384, False, False, "bf16"),   # logits: 256-wide pair tiles, TMA-stored bf16
    (3, 300, 512, 1000, False, True, "f32"),       # dX-like, partial pair tile
    (2, 1000, 768, 768, True, True, "f32"),        # weight-gradient shape
    (1, 512, 1024, 256, True, True, "f32"),        # N % 256 == 0 -> 256-wide pair tiles
    (2, 384, 2304, 320, True, False, "f32"),
    (2, 768, 1152, 384, False, False, "bf16"),
    (1, 256, 2560, 512, False, True, "bf16"),
    (2, 384, 384, 512, False, True, "f32"),        # N = 384: 192-wide pair tiles (64-byte-swizzled B halves)
    (2, 3072, 384, 4000, False, True, "f32"),      # LM-head input gradient shape
    (2, 4000, 384, 3072, True, True, "f32"),       # LM-head weight gradient shape, partial pair tile
    (1, 512, 576, 320, True, False, "f32"),        # 192-wide pair tiles with a K-major B
    (3, 300, 192, 200, False, True, "f32"),        # one 192-wide tile, partial M and K
])
def test_pair_gemm_matches_reference_and_single_cta(G, M, N, K, a_mn, b_mn, epi, monkeypatch):
    from opendipaco_b200.ops.gemm import gemm

    A = _bf(G, K, M, seed=1) if a_mn else _bf(G, M, K, seed=1)
    B = _bf(G, K, N, seed=2) if b_mn else _bf(G, N, K, seed=2)
    dt = torch.bfloat16 if epi == "bf16" else torch.float32
    lda = M if a_mn else K
    ldb = N if b_mn else K

    def run():
        C = torch.full((G, M, N), 7.0, device=DEV, dtype=dt)
        gemm(A, lda, M * K, a_mn, B, ldb, N * K, b_mn, C, N, M * N, M, N, K, G, epi)
        return C

    c_pair = _run(run, monkeypatch, True)
    c_one = _run(run, monkeypatch, False)
    a = A.float().transpose(1, 2) if a_mn else A.float()
    b = B.float() if b_mn else B.float().transpose(1, 2)
    ref = a @ b
    _close(c_pair, ref, 1e-2 if epi == "bf16" else 2e-3)
    _close(c_pair, c_one, 1e-2 if epi == "bf16" else 1e-5)


@pytest.mark.parametrize("G,M,N,K,a_mn,b_mn", [
    (2, 3072, 384, 4000, False, True),   # LM-head input gradient: dlogits x W
    (2, 4000, 384, 3072, True, True),    # LM-head weight gradient: dlogits^T x X
    (1, 300, 200, 640, False, False),    # partial tiles in M, N and K
    (3, 256, 576, 512, True, False),
])
def test_gemm_192_wide_tiles_match_reference(G, M, N, K, a_mn, b_mn, monkeypatch):
    """fp32-output GEMM on 128 x 192 tiles (TMEM: two 192-column accumulators in a
    512-column allocation) against fp32 PyTorch and against 128-wide tiles."""
    from opendipaco_b200.ops.gemm import gemm

    A = _bf(G, K, M, seed=3) if a_mn else _bf(G, M, K, seed=3)
    B = _bf(G, K, N, seed=4) if b_mn else _bf(G, N, K, seed=4)
    lda = M if a_mn else K
    ldb = N if b_mn else K
    outs = {}
    for bn in (192, 128):
        def run():
            C = torch.full((G, M, N), 7.0, device=DEV)
            gemm(A, lda, M * K, a_mn, B, ldb, N * K, b_mn, C, N, M * N, M, N, K, G, "f32", bn=bn)
            return C

        outs[bn] = _run(run, monkeypatch, False)
    a = A.float().transpose(1, 2) if a_mn else A.float()
    b = B.float() if b_mn else B.float().transpose(1, 2)
    _close(outs[192], a @ b, 2e-3)
    _close(outs[192], outs[128], 1e-5)


def _epi_case(epi, G, M, N, K, seed):
    """Operands and a call of one epilogue kind, returning its outputs."""
    from opendipaco_b200.ops.gemm import gemm

    if epi in ("f32", "f32_beta", "resid"):
        a, b = _bf(G, M, K, seed=seed), _bf(G, N, K, seed=seed + 1)
        r = torch.randn(G, M, N, generator=torch.Generator().manual_seed(seed)).to(DEV)

        def run():
            c = r.clone() if epi == "f32_beta" else torch.full((G, M, N), 5.0, device=DEV)
            gemm(a, K, M * K, False, b, K, N * K, False, c, N, M * N, M, N, K, G,
                 "resid" if epi == "resid" else "f32", bn=128, R=r if epi == "resid" else None, ldr=N, sr=M * N,
                 beta=0.5 if epi == "f32_beta" else 0.0)
            return (c,)
        return run
    Fd = N
    if epi == "swiglu":
        x, w = _bf(G, M, K, seed=seed), _bf(G, 2 * Fd, K, seed=seed + 1)

        def run():
            h = torch.zeros(G, M, Fd, device=DEV, dtype=torch.bfloat16)
            gu = torch.zeros(G, M, 2 * Fd, device=DEV, dtype=torch.bfloat16)
            gemm(x, K, M * K, False, w, K, 2 * Fd * K, False, h, Fd, M * Fd, M, 2 * Fd, K, G, "swiglu", bn=128,
                 aux=gu, ldx=2 * Fd, sx=M * 2 * Fd, f_half=Fd)
            return h, gu
        return run
    dy, wd = _bf(G, M, K, seed=seed), _bf(G, K, Fd, seed=seed + 1)
    gu = _bf(G, M, 2 * Fd, seed=seed + 2)

    def run():
        dgu = torch.zeros(G, M, 2 * Fd, device=DEV, dtype=torch.bfloat16)
        gemm(dy, K, M * K, False, wd, Fd, K * Fd, True, dgu, 2 * Fd, M * 2 * Fd, M, Fd, K, G, "swiglu_bwd", bn=128,
             aux=gu, ldx=2 * Fd, sx=M * 2 * Fd, f_half=Fd)
        return (dgu,)
    return run


@pytest.mark.parametrize("epi,G,M,N,K", [
    ("f32", 2, 300, 384, 256), ("f32", 1, 128, 200, 64), ("f32_beta", 2, 256, 384, 384),
    ("resid", 3, 300, 384, 1024), ("resid", 1, 100, 96, 128),
    ("swiglu", 2, 300, 1024, 384), ("swiglu", 1, 128, 96, 64),
    ("swiglu_bwd", 2, 300, 1024, 384), ("swiglu_bwd", 1, 200, 160, 128),
])
def test_tma_store_epilogues_match_per_thread_stores(epi, G, M, N, K, monkeypatch):
    """fp32 / residual / SwiGLU / SwiGLU-backward outputs staged in shared memory and
    written by TMA bulk stores (inputs TMA-loaded) equal the per-thread stores bit for bit,
    partial row and column tiles included."""
    run = _epi_case(epi, G, M, N, K, seed=21)
    for pair in (True, False):   # fp32 outputs with >= 256 rows take the CTA-pair kernel when allowed
        tma = _run(run, monkeypatch, pair)
        monkeypatch.setenv("ODP_GEMM_NO_TMA_STORE", "1")
        plain = _run(run, monkeypatch, pair)
        monkeypatch.delenv("ODP_GEMM_NO_TMA_STORE")
        for a, b in zip(tma, plain):
            assert torch.equal(a, b), (pair, (a.float() - b.float()).abs().max().item())


@pytest.mark.parametrize("S", [1, 2, 4, 8])
@pytest.mark.parametrize("G,M,N,K", [(2, 384, 384, 3072), (2, 1152, 384, 1024), (1, 320, 200, 512)])
def test_split_k_weight_gradient_matches_reference(S, G, M, N, K, monkeypatch):
    """Weight gradient C[g] = A[g] B[g]^T (both MN-major, K = tokens) split over K into S
    groups of one GEMM plus a fixed-order reduction: against fp32 PyTorch, against the
    unsplit GEMM, and its 32 x 32 box sums of squares against PyTorch's."""
    from opendipaco_b200.ops.gemm import gemm_wgrad

    monkeypatch.setenv("ODP_GEMM_2SM", "1")
    A = _bf(G, K, M, seed=5)
    B = _bf(G, K, N, seed=6)
    nb = ((M + 31) // 32) * ((N + 31) // 32)
    ws = torch.empty(G * S * M * N, device=DEV)

    def run(split):
        C = torch.full((G, M, N), 3.0, device=DEV)
        sq = torch.full((G, nb), -1.0, device=DEV)
        gemm_wgrad(A, M, K * M, B, N, K * N, C, N, M * N, M, N, K, G, split, ws, sq, nb)
        torch.cuda.synchronize()
        return C, sq

    if K % (64 * S):
        pytest.skip("K not divisible into 64-wide splits")
    c, sq = run(S)
    c1, _ = run(1)
    ref = A.float().transpose(1, 2) @ B.float()
    _close(c, ref, 2e-3)
    _close(c, c1, 1e-5)
    pad = torch.zeros(G, (M + 31) // 32 * 32, (N + 31) // 32 * 32, device=DEV)
    pad[:, :M, :N] = c
    boxes = pad.view(G, (M + 31) // 32, 32, (N + 31) // 32, 32).pow(2).sum((2, 4)).reshape(G, -1)
    _close(sq, boxes, 1e-4)
