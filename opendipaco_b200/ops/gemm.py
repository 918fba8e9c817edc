"""tcgen05 GEMM entry points (``csrc/gemm.cu``).

``gemm(A, B, ...)`` computes ``C[g] = A[g] @ B[g]^T`` for bf16 operands with fp32
accumulation. Each operand is described by (tensor, leading dim, group stride,
major): ``mn=False`` means the operand is stored ``[rows, K]`` (K contiguous),
``mn=True`` means it is stored ``[K, rows]``. Views into flat parameter buffers
are passed as (base tensor, offsets folded into a narrowed view).
"""

from __future__ import annotations

import os

import torch

from ._ext import err_word, ext

EPI = {"bf16": 0, "f32": 1, "resid": 2, "swiglu": 3, "swiglu_bwd": 4, "logits": 5}


def gemm(A, lda, sa, a_mn, B, ldb, sb, b_mn, C, ldc, sc, M, N, K, G=1, epi="bf16", bn=128, R=None, ldr=0,
         sr=0, aux=None, ldx=0, sx=0, part=None, beta=0.0, f_half=0, max_ctas=0, sq_part=None, sq_ld=0):
    ext().gemm_bf16(A, lda, sa, a_mn, B, ldb, sb, b_mn, C, ldc, sc, M, N, K, G, EPI[epi], bn, R, ldr, sr,
                    aux, ldx, sx, part, beta, f_half, err_word(A.device), max_ctas, sq_part, sq_ld)
    return C


def _bn_for(n: int) -> int:
    return 128 if n % 128 == 0 or n > 64 else 64


def mm_nt(a: torch.Tensor, b: torch.Tensor, out_dtype=torch.bfloat16, bn: int | None = None) -> torch.Tensor:
    """``a @ b.T`` with a: [M, K], b: [N, K] (both K-major)."""
    M, K = a.shape
    N = b.shape[0]
    c = torch.empty(M, N, device=a.device, dtype=out_dtype)
    gemm(a, a.stride(0), 0, False, b, b.stride(0), 0, False, c, c.stride(0), 0, M, N, K,
         epi="bf16" if out_dtype == torch.bfloat16 else "f32", bn=bn or _bn_for(N))
    return c


def mm_nn(a: torch.Tensor, b: torch.Tensor, out_dtype=torch.bfloat16, bn: int | None = None) -> torch.Tensor:
    """``a @ b`` with a: [M, K] (K-major), b: [K, N] (N contiguous -> MN-major operand)."""
    M, K = a.shape
    N = b.shape[1]
    c = torch.empty(M, N, device=a.device, dtype=out_dtype)
    gemm(a, a.stride(0), 0, False, b, b.stride(0), 0, True, c, c.stride(0), 0, M, N, K,
         epi="bf16" if out_dtype == torch.bfloat16 else "f32", bn=bn or _bn_for(N))
    return c


def mm_tn(a: torch.Tensor, b: torch.Tensor, out_dtype=torch.float32, bn: int | None = None) -> torch.Tensor:
    """``a.T @ b`` with a: [K, M], b: [K, N] (both MN-major) -- weight-gradient shape."""
    K, M = a.shape
    N = b.shape[1]
    c = torch.empty(M, N, device=a.device, dtype=out_dtype)
    gemm(a, a.stride(0), 0, True, b, b.stride(0), 0, True, c, c.stride(0), 0, M, N, K,
         epi="bf16" if out_dtype == torch.bfloat16 else "f32", bn=bn or _bn_for(N))
    return c


def mm_tt(a: torch.Tensor, b: torch.Tensor, out_dtype=torch.float32, bn: int | None = None) -> torch.Tensor:
    """``a.T @ b.T`` with a: [K, M] (MN-major), b: [N, K] (K-major)."""
    K, M = a.shape
    N = b.shape[0]
    c = torch.empty(M, N, device=a.device, dtype=out_dtype)
    gemm(a, a.stride(0), 0, True, b, b.stride(0), 0, False, c, c.stride(0), 0, M, N, K,
         epi="bf16" if out_dtype == torch.bfloat16 else "f32", bn=bn or _bn_for(N))
    return c


def sm_count(device=None) -> int:
    """Streaming multiprocessors of ``device`` (the current CUDA device by default); 148,
    a full B200, when no device is visible (CPU-side planning)."""
    if not torch.cuda.is_available():
        return 148
    d = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    return torch.cuda.get_device_properties(d).multi_processor_count


def splitk_factor(M: int, N: int, K: int, G: int, sms: int | None = None) -> int:
    """Number of K splits for a weight-gradient GEMM whose 128 x 128 output tiles leave
    most SMs idle: doubled while the split grid still fits one wave and each split keeps
    at least 384 of K in whole 64-wide k-blocks (``ODP_SPLITK`` forces a value). Only
    grids of at most an eighth of the SMs are split: measured at 2 paths per GPU, the
    extra reduction launch (~8 us) cancels the gain for grids of 48-54 tiles, while the
    18-tile attention-output gradient goes from 27 to 15 us."""
    sms = sm_count() if sms is None else sms
    forced = os.environ.get("ODP_SPLITK")
    tiles = G * ((M + 127) // 128) * ((N + 127) // 128)
    s = 1
    if forced:
        want = int(forced)
        while s < want and K % (2 * s * 64) == 0 and K // (2 * s) >= 64:
            s *= 2
        return s
    if tiles * 8 > sms:
        return 1
    while s < 8 and tiles * s * 2 <= sms and K % (2 * s * 64) == 0 and K // (2 * s) >= 384:
        s *= 2
    return s


def gemm_ce_wgrad(logits, ldl, sl, X, ldx, sx, C, ldc, sc, V, H, T, G, S, ws, ob, labels, scale, ms, sq_part=None,
                  sq_ld=0, err=None, beta=0.0):
    """LM-head weight gradient C[g] (V x H) = dlogits[g]^T X[g] with the dlogits formed from
    the bf16 logits inside the GEMM (``gemm_ce_grad``, mode 2); T tokens, split over them
    into S parts (workspace ``ws``, fixed-order reduction) like ``gemm_wgrad``."""
    x = ext()
    e = err if err is not None else err_word(logits.device)
    if S <= 1:
        x.gemm_ce_grad(logits, ldl, sl, True, X, ldx, sx, True, C, ldc, sc, V, H, T, G, beta, e, sq_part, sq_ld, 2, ob,
                       labels, scale, ms, 1)
        return C
    if sl != T * ldl or sx != T * ldx or T % (S * 64):
        raise ValueError("gemm_ce_wgrad: split-K needs contiguous groups along the tokens and T % (64 S) == 0")
    ts = T // S
    x.gemm_ce_grad(logits, ldl, ts * ldl, True, X, ldx, ts * ldx, True, ws, H, V * H, V, H, ts, G * S, 0.0, e, None, 0,
                   2, ob, labels, scale, ms, S)
    x.gemm_splitk_reduce(ws, S, G, V, H, C, ldc, sc, sq_part, sq_ld, beta)
    return C


def gemm_wgrad(A, lda, sa, B, ldb, sb, C, ldc, sc, M, N, K, G, S, ws, sq_part=None, sq_ld=0, err=None,
               beta=0.0, bn=128):
    """fp32 weight gradient C[g] = A[g] B[g]^T with both operands MN-major (K = tokens),
    split over K into S parts when S > 1: the splits run as G * S groups of one GEMM into
    the workspace ``ws`` and are summed in a fixed order by ``gemm_splitk_reduce`` (which
    also writes the 32 x 32 box sums of squares). Needs sa == K * lda and sb == K * ldb."""
    x = ext()
    e = err if err is not None else err_word(A.device)
    if S <= 1:
        x.gemm_bf16(A, lda, sa, True, B, ldb, sb, True, C, ldc, sc, M, N, K, G, EPI["f32"], bn, None, 0, 0,
                    None, 0, 0, None, beta, 0, e, 0, sq_part, sq_ld)
        return C
    if sa != K * lda or sb != K * ldb or K % (S * 64):
        raise ValueError("gemm_wgrad: split-K needs contiguous groups along K and K % (64 S) == 0")
    ks = K // S
    x.gemm_bf16(A, lda, ks * lda, True, B, ldb, ks * ldb, True, ws, N, M * N, M, N, ks, G * S, EPI["f32"], 128,
                None, 0, 0, None, 0, 0, None, 0.0, 0, e, 0, None, 0)
    x.gemm_splitk_reduce(ws, S, G, M, N, C, ldc, sc, sq_part, sq_ld, beta)
    return C
