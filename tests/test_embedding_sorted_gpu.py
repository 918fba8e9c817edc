"""Sort-based embedding backward (csrc/norm.cu embedding_bwd_sorted) against the
row-scan kernel (same additions in the same row order: bitwise equal) and an fp32
PyTorch reference, with Zipf-like repeated tokens and several paths."""

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("G,M,H,V", [(3, 3072, 384, 32000), (2, 1000, 64, 500), (1, 4096, 1024, 50000)])
def test_sorted_embedding_bwd(G, M, H, V):
    from opendipaco_b200.ops import check_errors
    from opendipaco_b200.ops._ext import ext

    g = torch.Generator(device="cpu").manual_seed(M)
    zipf = (torch.rand(G, M, generator=g) ** 4 * V).long().clamp_(0, V - 1)  # heavy head of repeats
    ids = zipf.to(torch.int32).to(DEV)
    dx = torch.randn(G, M, H, generator=g).to(DEV)
    a = torch.zeros(G, V, H, device=DEV)
    b = torch.zeros(G, V, H, device=DEV)
    keys = torch.zeros(G, M, dtype=torch.int32, device=DEV)
    ext().embedding_bwd(ids, dx, M * H, a, V * H, M, H, G, V)
    ext().embedding_bwd_sorted(ids, dx, M * H, b, V * H, M, H, G, V, keys, None, None)
    torch.cuda.synchronize()
    check_errors()
    assert torch.equal(a, b)
    for p in range(G):
        ref = torch.zeros(V, H, device=DEV).index_add_(0, zipf[p].to(DEV), dx[p])
        torch.testing.assert_close(b[p], ref, rtol=1e-5, atol=1e-4)
