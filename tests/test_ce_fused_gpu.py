"""One-pass cross-entropy (csrc/loss.cu ce_fused) against an fp32 PyTorch reference of
the same op: per-row log-sum-exp and loss, per-group mean loss, and dlogits =
(softmax - onehot) / valid-count written in place over the bf16 logits."""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("G,M,V", [(2, 96, 32000), (3, 50, 1000), (1, 7, 32768)])
def test_ce_fused_matches_fp32_reference(G, M, V):
    from opendipaco_b200.ops import check_errors
    from opendipaco_b200.ops._ext import err_word, ext

    g = torch.Generator(device="cpu").manual_seed(V)
    logits = (torch.randn(G, M, V, generator=g) * 3).to(DEV).to(torch.bfloat16)
    labels = torch.randint(0, V, (G, M), generator=g).to(DEV)
    labels[0, ::5] = -100
    lab32 = labels.to(torch.int32).reshape(-1).contiguous()
    lse, row_loss = torch.empty(G * M, device=DEV), torch.empty(G * M, device=DEV)
    loss_sum, inv, loss = torch.empty(G, device=DEV), torch.empty(G, device=DEV), torch.empty(G, device=DEV)
    x = logits.float().requires_grad_(True)
    ref_rows = F.cross_entropy(x.reshape(-1, V), labels.reshape(-1), ignore_index=-100, reduction="none")
    ref_loss = torch.stack([F.cross_entropy(x[i], labels[i], ignore_index=-100) for i in range(G)])
    ref_loss.sum().backward()
    d = logits.clone()
    ext().ce_fused(d, V, M * V, lab32, M, V, G, lse, row_loss, loss_sum, inv, loss, err_word(DEV), None)
    torch.cuda.synchronize()
    check_errors()
    torch.testing.assert_close(row_loss, ref_rows.detach(), rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(loss, ref_loss.detach(), rtol=1e-4, atol=1e-5)
    valid = (labels.reshape(-1) >= 0)
    torch.testing.assert_close(lse[valid], torch.logsumexp(x.reshape(-1, V), -1)[valid].detach(), rtol=1e-5,
                               atol=1e-4)
    ref_d = x.grad.to(torch.bfloat16).float()
    err = (d.float() - ref_d).abs().max().item()
    assert err <= 2e-2 * ref_d.abs().max().item(), err
    assert torch.all(d.reshape(-1, V)[~valid] == 0)
