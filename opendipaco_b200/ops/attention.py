"""Causal GQA attention with fused RoPE, head_dim 64.

Two kernel families: ``csrc/attention_tc.cu`` (tcgen05 + TMEM, one 128-row tile per
(sequence, head): used whenever S <= 128) and ``csrc/attention.cu`` (mma.sync, 64-row
blocks, any S that is a multiple of 64). ``ODP_ATTN_IMPL=mma`` forces the latter.
"""

from __future__ import annotations

import os

import torch

from ._ext import err_word, ext

TC_MAX_S = 128


def use_tc(S: int) -> bool:
    impl = os.environ.get("ODP_ATTN_IMPL", "auto")
    return impl != "mma" and S <= TC_MAX_S


def fwd(qkv, GB, S, nh, nkv, cos, sin, o, lse, err=None) -> None:
    """Launch the forward kernel on preallocated outputs (no allocation)."""
    if use_tc(S):
        ext().attention_fwd_tc(qkv, GB, S, nh, nkv, cos, sin, o, lse, err if err is not None else err_word(qkv.device))
    else:
        ext().attention_fwd(qkv, GB, S, nh, nkv, cos, sin, o, lse)


def bwd(qkv, GB, S, nh, nkv, cos, sin, o, lse, dout, delta, dqkv, err=None) -> None:
    """Launch the backward kernels on preallocated buffers (``delta`` is scratch of the
    mma.sync path; the tcgen05 path computes it in the kernel)."""
    if use_tc(S):
        ext().attention_bwd_tc(qkv, GB, S, nh, nkv, cos, sin, o, lse, dout, dqkv,
                               err if err is not None else err_word(qkv.device))
    else:
        ext().attention_bwd(qkv, GB, S, nh, nkv, cos, sin, o, lse, dout, delta, dqkv)


def attention_fwd(qkv: torch.Tensor, nh: int, nkv: int, cos: torch.Tensor, sin: torch.Tensor):
    """qkv: [B, S, (nh+2nkv)*64] bf16 (q|k|v, pre-RoPE) -> (o [B, S, nh*64] bf16, lse [B, nh, S])."""
    B, S, C = qkv.shape
    assert C == (nh + 2 * nkv) * 64 and (S <= TC_MAX_S or S % 64 == 0)
    o = torch.empty(B, S, nh * 64, device=qkv.device, dtype=torch.bfloat16)
    lse = torch.empty(B, nh, S, device=qkv.device, dtype=torch.float32)
    fwd(qkv, B, S, nh, nkv, cos, sin, o, lse)
    return o, lse


def attention_bwd(qkv, o, lse, dout, nh, nkv, cos, sin):
    """Returns dqkv [B, S, (nh+2nkv)*64] bf16 (gradient w.r.t. the pre-RoPE q|k|v)."""
    B, S, C = qkv.shape
    dqkv = torch.empty_like(qkv)
    delta = torch.empty(B, nh, S, device=qkv.device, dtype=torch.float32)
    bwd(qkv, B, S, nh, nkv, cos, sin, o, lse, dout.contiguous(), delta, dqkv)
    return dqkv
