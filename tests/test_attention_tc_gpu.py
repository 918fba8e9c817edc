"""tcgen05 attention (csrc/attention_tc.cu) against an fp32 PyTorch reference of the same
op (RoPE + causal softmax attention, GQA) and against the mma.sync kernels."""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
DEV = "cuda"
D = 64


def _bf(*shape, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randn(*shape, generator=g).to(DEV).to(torch.bfloat16)


def _close(a, b, tol):
    a, b = a.float(), b.float()
    err = (a - b).abs().max().item()
    ref = b.abs().max().item() + 1e-6
    assert err <= tol * ref, f"max err {err} vs ref max {ref} (tol {tol})"


def _rope(x, cos, sin):
    h = x.shape[-1] // 2
    return x * cos + torch.cat([-x[..., h:], x[..., :h]], -1) * sin


def _reference(qkv, nh, nkv, cos, sin):
    B, S, _ = qkv.shape
    x = qkv.float().requires_grad_(True)
    q = x[..., :nh * D].view(B, S, nh, D).transpose(1, 2)
    k = x[..., nh * D:(nh + nkv) * D].view(B, S, nkv, D).transpose(1, 2)
    v = x[..., (nh + nkv) * D:].view(B, S, nkv, D).transpose(1, 2)
    q, k = _rope(q, cos, sin), _rope(k, cos, sin)
    k, v = k.repeat_interleave(nh // nkv, 1), v.repeat_interleave(nh // nkv, 1)
    o = F.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(1, 2).reshape(B, S, nh * D)
    return x, o


def _run(impl, qkv, nh, nkv, cos, sin, do, monkeypatch):
    from opendipaco_b200.ops import check_errors
    from opendipaco_b200.ops.attention import attention_bwd, attention_fwd

    monkeypatch.setenv("ODP_ATTN_IMPL", impl)
    o, lse = attention_fwd(qkv, nh, nkv, cos, sin)
    dqkv = attention_bwd(qkv, o, lse, do, nh, nkv, cos, sin)
    torch.cuda.synchronize()
    check_errors()
    return o, lse, dqkv


@pytest.mark.parametrize("B,S,nh,nkv", [(3, 128, 6, 6), (2, 100, 8, 2), (4, 64, 4, 4), (2, 37, 4, 1)])
def test_tc_attention_matches_fp32_reference(B, S, nh, nkv, monkeypatch):
    from opendipaco_b200.models.llama import rope_cos_sin
    from opendipaco_b200.ops.attention import use_tc

    assert use_tc(S)
    cos, sin = rope_cos_sin(D, 10000.0, S, DEV)
    qkv = _bf(B, S, (nh + 2 * nkv) * D, seed=S)
    do = _bf(B, S, nh * D, seed=S + 1)
    o, lse, dqkv = _run("auto", qkv, nh, nkv, cos, sin, do, monkeypatch)
    x, ref = _reference(qkv, nh, nkv, cos, sin)
    _close(o, ref, 2e-2)
    ref.backward(do.float())
    _close(dqkv, x.grad, 3e-2)
    # log-sum-exp of the scaled causal scores
    q = _rope(qkv.float()[..., :nh * D].view(B, S, nh, D).transpose(1, 2), cos, sin)
    k = _rope(qkv.float()[..., nh * D:(nh + nkv) * D].view(B, S, nkv, D).transpose(1, 2), cos, sin)
    s = (q @ k.repeat_interleave(nh // nkv, 1).transpose(-1, -2)) / D ** 0.5
    s = s.masked_fill(torch.ones(S, S, device=DEV, dtype=torch.bool).triu(1), float("-inf"))
    _close(lse, torch.logsumexp(s, -1), 1e-2)


@pytest.mark.parametrize("S", [128, 64])
def test_tc_attention_matches_mma_kernels(S, monkeypatch):
    from opendipaco_b200.models.llama import rope_cos_sin

    B, nh, nkv = 4, 6, 3
    cos, sin = rope_cos_sin(D, 10000.0, S, DEV)
    qkv = _bf(B, S, (nh + 2 * nkv) * D, seed=7)
    do = _bf(B, S, nh * D, seed=8)
    o1, l1, d1 = _run("auto", qkv, nh, nkv, cos, sin, do, monkeypatch)
    o2, l2, d2 = _run("mma", qkv, nh, nkv, cos, sin, do, monkeypatch)
    _close(o1, o2, 1e-2)
    _close(l1, l2, 1e-4)
    _close(d1, d2, 2e-2)


def test_tc_attention_is_deterministic(monkeypatch):
    from opendipaco_b200.models.llama import rope_cos_sin

    B, S, nh, nkv = 2, 128, 4, 2
    cos, sin = rope_cos_sin(D, 10000.0, S, DEV)
    qkv = _bf(B, S, (nh + 2 * nkv) * D, seed=3)
    do = _bf(B, S, nh * D, seed=4)
    a = _run("auto", qkv, nh, nkv, cos, sin, do, monkeypatch)
    b = _run("auto", qkv, nh, nkv, cos, sin, do, monkeypatch)
    for x, y in zip(a, b):
        assert torch.equal(x, y)


# ---------------------------------------------------------------- S > 128: flash kernels
def _lse_ref(qkv, nh, nkv, cos, sin):
    B, S, _ = qkv.shape
    q = _rope(qkv.float()[..., :nh * D].view(B, S, nh, D).transpose(1, 2), cos, sin)
    k = _rope(qkv.float()[..., nh * D:(nh + nkv) * D].view(B, S, nkv, D).transpose(1, 2), cos, sin)
    s = (q @ k.repeat_interleave(nh // nkv, 1).transpose(-1, -2)) / D ** 0.5
    s = s.masked_fill(torch.ones(S, S, device=DEV, dtype=torch.bool).triu(1), float("-inf"))
    return torch.logsumexp(s, -1)


@pytest.mark.parametrize("B,S,nh,nkv", [(1, 256, 32, 8), (1, 512, 32, 8), (1, 1024, 32, 8), (2, 200, 4, 1),
                                        (2, 320, 6, 6)])
def test_flash_attention_matches_fp32_reference(B, S, nh, nkv, monkeypatch):
    """Long sequences (GQA 32 query / 8 kv heads as in the 1B Llama shape, a ragged S = 200
    with one kv head, a 64-multiple S = 320 without GQA) against fp32 SDPA."""
    from opendipaco_b200.models.llama import rope_cos_sin
    from opendipaco_b200.ops.attention import impl_for

    assert impl_for(S) == "flash"
    cos, sin = rope_cos_sin(D, 10000.0, S, DEV)
    qkv = _bf(B, S, (nh + 2 * nkv) * D, seed=S + nh)
    do = _bf(B, S, nh * D, seed=S + nh + 1)
    o, lse, dqkv = _run("auto", qkv, nh, nkv, cos, sin, do, monkeypatch)
    x, ref = _reference(qkv, nh, nkv, cos, sin)
    _close(o, ref, 2e-2)
    _close(lse, _lse_ref(qkv, nh, nkv, cos, sin), 1e-2)
    ref.backward(do.float())
    _close(dqkv, x.grad, 3e-2)
    # each of q, k and v gradients on its own scale (k and v sum over GQA heads)
    for lo, hi in ((0, nh * D), (nh * D, (nh + nkv) * D), ((nh + nkv) * D, (nh + 2 * nkv) * D)):
        _close(dqkv[..., lo:hi], x.grad[..., lo:hi], 3e-2)


def test_flash_attention_matches_mma_kernels(monkeypatch):
    from opendipaco_b200.models.llama import rope_cos_sin

    B, S, nh, nkv = 2, 512, 8, 2
    cos, sin = rope_cos_sin(D, 10000.0, S, DEV)
    qkv = _bf(B, S, (nh + 2 * nkv) * D, seed=11)
    do = _bf(B, S, nh * D, seed=12)
    o1, l1, d1 = _run("auto", qkv, nh, nkv, cos, sin, do, monkeypatch)
    o2, l2, d2 = _run("mma", qkv, nh, nkv, cos, sin, do, monkeypatch)
    _close(o1, o2, 1e-2)
    _close(l1, l2, 1e-4)
    _close(d1, d2, 2e-2)


def test_flash_attention_is_deterministic(monkeypatch):
    from opendipaco_b200.models.llama import rope_cos_sin

    B, S, nh, nkv = 2, 384, 8, 2
    cos, sin = rope_cos_sin(D, 10000.0, S, DEV)
    qkv = _bf(B, S, (nh + 2 * nkv) * D, seed=5)
    do = _bf(B, S, nh * D, seed=6)
    a = _run("auto", qkv, nh, nkv, cos, sin, do, monkeypatch)
    b = _run("auto", qkv, nh, nkv, cos, sin, do, monkeypatch)
    for x, y in zip(a, b):
        assert torch.equal(x, y)


@pytest.mark.parametrize("B,S,nh,nkv", [(2, 200, 4, 1), (1, 384, 8, 2)])
def test_flash_rotation_pass_gives_the_same_bits(B, S, nh, nkv):
    """q|k rotated once into a scratch by a separate pass, or in every staged tile: the
    same rotation code on the same bits, so forward and backward agree exactly."""
    from opendipaco_b200.models.llama import rope_cos_sin
    from opendipaco_b200.ops import attention as attn
    from opendipaco_b200.ops import check_errors

    cos, sin = rope_cos_sin(D, 10000.0, S, DEV)
    qkv = _bf(B, S, (nh + 2 * nkv) * D, seed=7)
    do = _bf(B, S, nh * D, seed=8)
    outs = []
    for use in (False, True):
        o = torch.empty(B, S, nh * D, device=DEV, dtype=torch.bfloat16)
        lse = torch.empty(B, nh, S, device=DEV)
        delta = torch.empty(B, nh, S, device=DEV)
        dqkv = torch.zeros_like(qkv)
        qkr = torch.empty(attn.qkr_shape(B, S, nh, nkv), device=DEV, dtype=torch.bfloat16) if use else None
        attn.fwd(qkv, B, S, nh, nkv, cos, sin, o, lse, qkr=qkr)
        attn.bwd(qkv, B, S, nh, nkv, cos, sin, o, lse, do, delta, dqkv, qkr=qkr)
        torch.cuda.synchronize()
        check_errors()
        outs.append((o, lse, dqkv))
    for x, y in zip(*outs):
        assert torch.equal(x, y)
