"""Causal GQA attention with fused RoPE, head_dim 64, on the tcgen05 tensor cores.

Two kernel families in ``csrc/attention_tc.cu``, both tcgen05 + TMEM with RoPE applied
while the tiles are staged:

* S <= 128: one 128-row tile per (sequence, head) (``attention_{fwd,bwd}_tc``);
* S > 128: flash kernels (``attention_{fwd,bwd}_flash``) -- online softmax over 64-key
  tiles in the forward, a dQ kernel (which also writes delta = rowsum(dO o)) and an
  atomic-free dK / dV kernel in the backward.

``ODP_ATTN_IMPL=mma`` selects the older ``mma.sync`` kernels of ``csrc/attention.cu``
(S a multiple of 64) instead, for comparison only; no training path uses them otherwise.
The reference computes the same op with ``F.scaled_dot_product_attention(is_causal=True)``
after HF-style RoPE (``src/opendipaco/modules.py:38``).
"""

from __future__ import annotations

import os

import torch

from ._ext import err_word, ext

TC_MAX_S = 128


def impl_for(S: int) -> str:
    """Kernel family used for sequence length S: "tc" (one tile), "flash" or "mma"."""
    if os.environ.get("ODP_ATTN_IMPL", "auto") == "mma":
        return "mma"
    return "tc" if S <= TC_MAX_S else "flash"


def use_tc(S: int) -> bool:
    return impl_for(S) != "mma"


def qkr_shape(GB: int, S: int, nh: int, nkv: int) -> tuple | None:
    """Shape of the rotated-q|k scratch the flash kernels take (None: not used for S)."""
    return (GB, S, (nh + nkv) * 64) if impl_for(S) == "flash" else None


def fwd(qkv, GB, S, nh, nkv, cos, sin, o, lse, err=None, qkr=None) -> None:
    """Launch the forward kernel on preallocated outputs (no allocation). Flash path: with
    ``qkr`` (bf16 ``qkr_shape``) q|k are rotated once into it, else in every staged tile."""
    impl = impl_for(S)
    e = err if err is not None else err_word(qkv.device)
    if impl == "tc":
        ext().attention_fwd_tc(qkv, GB, S, nh, nkv, cos, sin, o, lse, e)
    elif impl == "flash":
        ext().attention_fwd_flash(qkv, GB, S, nh, nkv, cos, sin, o, lse, e, qkr)
    else:
        ext().attention_fwd(qkv, GB, S, nh, nkv, cos, sin, o, lse)


def bwd(qkv, GB, S, nh, nkv, cos, sin, o, lse, dout, delta, dqkv, err=None, qkr=None) -> None:
    """Launch the backward kernels on preallocated buffers. ``delta`` [GB, nh, S] fp32
    receives rowsum(dO o) (flash and mma paths); the one-tile kernel computes it in
    registers and leaves ``delta`` untouched. ``qkr`` as in :func:`fwd`."""
    impl = impl_for(S)
    e = err if err is not None else err_word(qkv.device)
    if impl == "tc":
        ext().attention_bwd_tc(qkv, GB, S, nh, nkv, cos, sin, o, lse, dout, dqkv, e)
    elif impl == "flash":
        ext().attention_bwd_flash(qkv, GB, S, nh, nkv, cos, sin, o, lse, dout, delta, dqkv, e, qkr)
    else:
        ext().attention_bwd(qkv, GB, S, nh, nkv, cos, sin, o, lse, dout, delta, dqkv)


def attention_fwd(qkv: torch.Tensor, nh: int, nkv: int, cos: torch.Tensor, sin: torch.Tensor):
    """qkv: [B, S, (nh+2nkv)*64] bf16 (q|k|v, pre-RoPE) -> (o [B, S, nh*64] bf16, lse [B, nh, S])."""
    B, S, C = qkv.shape
    assert C == (nh + 2 * nkv) * 64 and (impl_for(S) != "mma" or S % 64 == 0)
    o = torch.empty(B, S, nh * 64, device=qkv.device, dtype=torch.bfloat16)
    lse = torch.empty(B, nh, S, device=qkv.device, dtype=torch.float32)
    shp = qkr_shape(B, S, nh, nkv)
    qkr = torch.empty(shp, device=qkv.device, dtype=torch.bfloat16) if shp else None
    fwd(qkv, B, S, nh, nkv, cos, sin, o, lse, qkr=qkr)
    return o, lse


def attention_bwd(qkv, o, lse, dout, nh, nkv, cos, sin):
    """Returns dqkv [B, S, (nh+2nkv)*64] bf16 (gradient w.r.t. the pre-RoPE q|k|v)."""
    B, S, C = qkv.shape
    dqkv = torch.empty_like(qkv)
    delta = torch.empty(B, nh, S, device=qkv.device, dtype=torch.float32)
    shp = qkr_shape(B, S, nh, nkv)
    qkr = torch.empty(shp, device=qkv.device, dtype=torch.bfloat16) if shp else None
    bwd(qkv, B, S, nh, nkv, cos, sin, o, lse, dout.contiguous(), delta, dqkv, qkr=qkr)
    return dqkv
