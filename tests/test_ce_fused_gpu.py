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


@pytest.mark.parametrize("G,M,V,H,S", [(2, 3072, 32000, 384, 1), (2, 300, 1000, 256, 1), (1, 512, 2048, 384, 2)])
def test_ce_gradient_gemms_equal_in_place_dlogits_bitwise(G, M, V, H, S):
    """The LM-head gradient GEMMs that form the dlogits from the logits while staging their
    operand give the same bits as the in-place CE pass followed by the plain GEMMs: input
    gradient (K = vocab), weight gradient (K = tokens; S > 1: split over the tokens),
    ignored labels, partial tiles."""
    from opendipaco_b200.ops import check_errors
    from opendipaco_b200.ops._ext import err_word, ext
    from opendipaco_b200.ops.gemm import gemm_ce_wgrad, gemm_wgrad

    g = torch.Generator(device="cpu").manual_seed(M + V)
    logits = (torch.randn(G, M, V, generator=g) * 3).to(DEV).to(torch.bfloat16)
    labels = torch.randint(0, V, (G, M), generator=g).to(DEV).to(torch.int32)
    labels[0, ::7] = -100
    lab = labels.reshape(-1).contiguous()
    W = (torch.randn(V, H, generator=g) * 0.05).to(DEV).to(torch.bfloat16)  # lm_head weight, one per group
    Wg = W.unsqueeze(0).expand(G, V, H).contiguous()
    X = (torch.randn(G, M, H, generator=g)).to(DEV).to(torch.bfloat16)
    err = err_word(DEV)
    mk = lambda *s: torch.empty(*s, device=DEV)  # noqa: E731
    lse, rows, lsum, inv, loss = mk(G * M), mk(G * M), mk(G), mk(G), mk(G)
    # reference: in-place dlogits, then the plain fp32 GEMMs
    d = logits.clone()
    ext().ce_fused(d, V, M * V, lab, M, V, G, lse, rows, lsum, inv, loss, err, None)
    dx_ref, dw_ref = torch.zeros(G, M, H, device=DEV), torch.zeros(G, V, H, device=DEV)
    from opendipaco_b200.ops.gemm import EPI

    ext().gemm_bf16(d, V, M * V, False, Wg, H, V * H, True, dx_ref, H, M * H, M, H, V, G, EPI["f32"], 128, None, 0,
                    0, None, 0, 0, None, 0.0, 0, err, 0, None, 0)
    ws = torch.empty(G * S * V * H, device=DEV)
    gemm_wgrad(d, V, M * V, X, H, M * H, dw_ref, H, V * H, V, H, M, G, S, ws, err=err)
    # fused: the logits stay untouched; ob per row from the read-only CE pass
    ob, lse2, rows2, lsum2, inv2, loss2 = mk(G * M), mk(G * M), mk(G * M), mk(G), mk(G), mk(G)
    keep = logits.clone()
    ext().ce_fused(keep, V, M * V, lab, M, V, G, lse2, rows2, lsum2, inv2, loss2, err, None, ob)
    assert torch.equal(keep, logits) and torch.equal(loss2, loss) and torch.equal(lse2, lse)
    dx, dw = torch.zeros_like(dx_ref), torch.zeros_like(dw_ref)
    ext().gemm_ce_grad(keep, V, M * V, False, Wg, H, V * H, True, dx, H, M * H, M, H, V, G, 0.0, err, None, 0, 1, ob,
                       lab, inv2, M, 1)
    gemm_ce_wgrad(keep, V, M * V, X, H, M * H, dw, H, V * H, V, H, M, G, S, ws, ob, lab, inv2, M, err=err)
    torch.cuda.synchronize()
    check_errors()
    assert torch.equal(dx, dx_ref)
    assert torch.equal(dw, dw_ref)
