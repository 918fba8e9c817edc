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
    (2, 384, 384, 512, False, True, "f32"),        # narrow N: single-CTA kernel either way
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
