"""Autograd functions that run the nn.Module path on the sm_100a kernels.

Used when a :class:`~opendipaco_b200.models.path.PathModel` runs on CUDA outside the
fused executor (evaluation, routed perplexity, EM scoring, featurizers, or training
with ``ExecOptions(fused=False)``). Numerics follow bf16 autocast: GEMM operands in
bf16 with fp32 accumulation, the residual stream and RMSNorm statistics in fp32.
Sequences whose length is not a multiple of 64 are zero-padded at the end for the
attention kernel (causal masking makes the padding invisible to real positions).
"""

from __future__ import annotations

import torch

from . import attention as attn
from ._ext import err_word, ext
from .gemm import EPI


def _g(A, lda, amn, B, ldb, bmn, C, ldc, M, N, K, epi="bf16", bn=None, **kw):
    tiles = ((M + 127) // 128) * ((N + 127) // 128)
    ext().gemm_bf16(A, lda, 0, amn, B, ldb, 0, bmn, C, ldc, 0, M, N, K, 1, EPI[epi],
                    bn or (128 if tiles >= 148 else 64), kw.get("R"), kw.get("ldr", 0), 0, kw.get("aux"),
                    kw.get("ldx", 0), 0, kw.get("part"), kw.get("beta", 0.0), kw.get("f_half", 0),
                    err_word(A.device), 0, None, 0)
    return C


def _bf(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).contiguous()


# ---------------------------------------------------------------------- linear
class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, out_f32):
        x16, w16 = _bf(x.reshape(-1, x.shape[-1])), _bf(w)
        R, K = x16.shape
        N = w16.shape[0]
        y = torch.empty(R, N, device=x.device, dtype=torch.float32 if out_f32 else torch.bfloat16)
        _g(x16, K, False, w16, K, False, y, N, R, N, K, "f32" if out_f32 else "bf16")
        ctx.save_for_backward(x16, w16)
        ctx.shape = x.shape
        return y.view(*x.shape[:-1], N)

    @staticmethod
    def backward(ctx, dy):
        x16, w16 = ctx.saved_tensors
        R, K = x16.shape
        N = w16.shape[0]
        dy16 = _bf(dy.reshape(R, N))
        dx = torch.empty(R, K, device=dy.device, dtype=torch.float32)
        _g(dy16, N, False, w16, K, True, dx, K, R, K, N, "f32")
        dw = torch.empty(N, K, device=dy.device, dtype=torch.float32)
        _g(dy16, N, True, x16, K, True, dw, K, N, K, R, "f32")
        return dx.view(ctx.shape), dw, None


def linear(x: torch.Tensor, w: torch.Tensor, out_f32: bool = False) -> torch.Tensor:
    return _Linear.apply(x, w, out_f32)


# ---------------------------------------------------------------------- RMSNorm
class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        xf = x.float().reshape(-1, x.shape[-1]).contiguous()
        R, H = xf.shape
        y = torch.empty(R, H, device=x.device, dtype=torch.bfloat16)
        rstd = torch.empty(R, device=x.device, dtype=torch.float32)
        ext().rmsnorm_fwd(xf, 0, w.float().contiguous(), 0, y, 0, rstd, R, H, 1, eps)
        ctx.save_for_backward(xf, w, rstd)
        ctx.shape = x.shape
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, dy):
        xf, w, rstd = ctx.saved_tensors
        R, H = xf.shape
        dx = torch.empty_like(xf)
        dw = torch.empty(H, device=xf.device, dtype=torch.float32)
        work = torch.empty(((R + 31) // 32) * H, device=xf.device, dtype=torch.float32)
        ext().rmsnorm_bwd(xf, 0, w.float().contiguous(), 0, rstd, dy.float().reshape(R, H).contiguous(), 0,
                          None, dx, 0, None, dw, 0, work, R, H, 1, 0.0)
        return dx.view(ctx.shape), dw, None


def rms_norm(x, w, eps):
    if x.shape[-1] % 128:
        raise ValueError("CUDA RMSNorm kernel needs hidden % 128 == 0")
    return _RMSNorm.apply(x, w, eps)


# ---------------------------------------------------------------------- embedding
class _Embedding(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, w):
        ids32 = ids.reshape(-1).to(torch.int32).contiguous()
        V, H = w.shape
        out = torch.empty(ids32.numel(), H, device=w.device, dtype=torch.float32)
        ext().embedding_fwd(ids32, w.float().contiguous(), 0, out, ids32.numel(), H, 1, V)
        ctx.save_for_backward(ids32)
        ctx.V = V
        return out.view(*ids.shape, H)

    @staticmethod
    def backward(ctx, dy):
        (ids32,) = ctx.saved_tensors
        H = dy.shape[-1]
        dE = torch.zeros(ctx.V, H, device=dy.device, dtype=torch.float32)
        ext().embedding_bwd(ids32, dy.float().reshape(-1, H).contiguous(), 0, dE, 0, ids32.numel(), H, 1, ctx.V)
        return None, dE


def embedding(ids, w):
    return _Embedding.apply(ids, w)


# ---------------------------------------------------------------------- attention core
class _AttnCore(torch.autograd.Function):
    """qkv [b, s, (nh+2nkv)*64] bf16 (pre-RoPE) -> o [b, s, nh*64] bf16."""

    @staticmethod
    def forward(ctx, qkv, nh, nkv, theta):
        from ..models.llama import rope_cos_sin

        b, s, c = qkv.shape
        sp = s if attn.use_tc(s) else (s + 63) // 64 * 64  # the tcgen05 kernel masks any S <= 128
        q = qkv if sp == s else torch.nn.functional.pad(qkv, (0, 0, 0, sp - s))
        q = q.contiguous()
        cos, sin = rope_cos_sin(64, theta, sp, qkv.device)
        o = torch.empty(b, sp, nh * 64, device=qkv.device, dtype=torch.bfloat16)
        lse = torch.empty(b, nh, sp, device=qkv.device, dtype=torch.float32)
        attn.fwd(q, b, sp, nh, nkv, cos, sin, o, lse)
        ctx.save_for_backward(q, o, lse, cos, sin)
        ctx.meta = (nh, nkv, s, sp)
        return o[:, :s]

    @staticmethod
    def backward(ctx, do):
        q, o, lse, cos, sin = ctx.saved_tensors
        nh, nkv, s, sp = ctx.meta
        b = q.shape[0]
        dop = torch.zeros(b, sp, nh * 64, device=do.device, dtype=torch.bfloat16)
        dop[:, :s] = do.to(torch.bfloat16)
        dq = torch.empty_like(q)
        delta = torch.empty(b, nh, sp, device=q.device, dtype=torch.float32)
        attn.bwd(q, b, sp, nh, nkv, cos, sin, o, lse, dop, delta, dq)
        return dq[:, :s], None, None, None


def attention_block(x, mod, cos, sin, pad_mask=None):
    if pad_mask is not None:
        raise NotImplementedError("key-padding masks are not supported by the CUDA attention kernel; "
                                  "right-pad and rely on causal masking")
    if mod.head_dim != 64:
        raise ValueError("CUDA attention kernel needs head_dim 64")
    w = torch.cat([mod.q_proj.weight, mod.k_proj.weight, mod.v_proj.weight], 0)
    qkv = linear(x, w)
    theta = getattr(mod, "rope_theta", None)
    if theta is None:
        # recover theta from the sin/cos table: cos(pos * theta^(-2i/d)); use i = 1
        theta = 10000.0
    o = _AttnCore.apply(qkv, mod.num_heads, mod.num_kv, theta)
    return linear(o, mod.o_proj.weight, out_f32=True)


# ---------------------------------------------------------------------- SwiGLU MLP
class _MLP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, wg, wu, wd):
        x16 = _bf(x.reshape(-1, x.shape[-1]))
        R, H = x16.shape
        Fd = wg.shape[0]
        wgu = _bf(torch.cat([wg, wu], 0))
        wd16 = _bf(wd)
        act = torch.empty(R, Fd, device=x.device, dtype=torch.bfloat16)
        gu = torch.empty(R, 2 * Fd, device=x.device, dtype=torch.bfloat16)
        _g(x16, H, False, wgu, H, False, act, Fd, R, 2 * Fd, H, "swiglu", bn=128, aux=gu, ldx=2 * Fd, f_half=Fd)
        out = torch.empty(R, H, device=x.device, dtype=torch.float32)
        _g(act, Fd, False, wd16, Fd, False, out, H, R, H, Fd, "f32")
        ctx.save_for_backward(x16, wgu, wd16, gu, act)
        ctx.shape = x.shape
        return out.view(x.shape)

    @staticmethod
    def backward(ctx, dout):
        x16, wgu, wd16, gu, act = ctx.saved_tensors
        R, H = x16.shape
        Fd = wd16.shape[1]
        dy16 = _bf(dout.reshape(R, H))
        dgu = torch.empty(R, 2 * Fd, device=dout.device, dtype=torch.bfloat16)
        _g(dy16, H, False, wd16, Fd, True, dgu, 2 * Fd, R, Fd, H, "swiglu_bwd", aux=gu, ldx=2 * Fd, f_half=Fd)
        dwd = torch.empty(H, Fd, device=dout.device, dtype=torch.float32)
        _g(dy16, H, True, act, Fd, True, dwd, Fd, H, Fd, R, "f32")
        dx = torch.empty(R, H, device=dout.device, dtype=torch.float32)
        _g(dgu, 2 * Fd, False, wgu, H, True, dx, H, R, H, 2 * Fd, "f32")
        dwgu = torch.empty(2 * Fd, H, device=dout.device, dtype=torch.float32)
        _g(dgu, 2 * Fd, True, x16, H, True, dwgu, H, 2 * Fd, H, R, "f32")
        return dx.view(ctx.shape), dwgu[:Fd], dwgu[Fd:], dwd


def mlp_block(x, mod):
    return _MLP.apply(x, mod.gate_proj.weight, mod.up_proj.weight, mod.down_proj.weight)
