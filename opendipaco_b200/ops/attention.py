"""Causal GQA attention with fused RoPE (``csrc/attention.cu``), head_dim 64."""

from __future__ import annotations

import torch

from ._ext import ext


def attention_fwd(qkv: torch.Tensor, nh: int, nkv: int, cos: torch.Tensor, sin: torch.Tensor):
    """qkv: [B, S, (nh+2nkv)*64] bf16 (q|k|v, pre-RoPE) -> (o [B, S, nh*64] bf16, lse [B, nh, S])."""
    B, S, C = qkv.shape
    assert C == (nh + 2 * nkv) * 64 and S % 64 == 0
    o = torch.empty(B, S, nh * 64, device=qkv.device, dtype=torch.bfloat16)
    lse = torch.empty(B, nh, S, device=qkv.device, dtype=torch.float32)
    ext().attention_fwd(qkv, B, S, nh, nkv, cos, sin, o, lse)
    return o, lse


def attention_bwd(qkv, o, lse, dout, nh, nkv, cos, sin):
    """Returns dqkv [B, S, (nh+2nkv)*64] bf16 (gradient w.r.t. the pre-RoPE q|k|v)."""
    B, S, C = qkv.shape
    dqkv = torch.empty_like(qkv)
    delta = torch.empty(B, nh, S, device=qkv.device, dtype=torch.float32)
    ext().attention_bwd(qkv, B, S, nh, nkv, cos, sin, o, lse, dout.contiguous(), delta, dqkv)
    return dqkv
