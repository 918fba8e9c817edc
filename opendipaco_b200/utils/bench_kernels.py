"""Device-timed micro-benchmarks of the hot kernels at the shapes of one fused training
step (CUDA events on the launching stream, warm-up first, L2 flushed between timed
launches by writing a 256 MB buffer), printed as one JSON line per case.

    python -m opendipaco_b200.utils.bench_kernels [--paths 16] [--only attention]

Default shapes: 16 paths x 24 sequences x 128 tokens, hidden 384, 6 heads, vocab 32000.
"""

from __future__ import annotations

import argparse
import json
import os

import torch


def _timeit(fn, reps: int, flush: torch.Tensor) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(reps):
        flush.add_(1.0)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        total += a.elapsed_time(b)
    return total / reps


def bench_attention(GB: int, S: int, nh: int, nkv: int, reps: int, flush) -> list[dict]:
    from ..models.llama import rope_cos_sin
    from ..ops import attention as attn
    from ..ops._ext import check_errors

    dev = torch.device("cuda")
    D = 64
    cos, sin = rope_cos_sin(D, 10000.0, S, dev)
    qkv = torch.randn(GB, S, (nh + 2 * nkv) * D, device=dev).to(torch.bfloat16)
    do = torch.randn(GB, S, nh * D, device=dev).to(torch.bfloat16)
    o = torch.empty(GB, S, nh * D, device=dev, dtype=torch.bfloat16)
    lse = torch.empty(GB, nh, S, device=dev)
    delta = torch.empty(GB, nh, S, device=dev)
    dqkv = torch.empty_like(qkv)
    out = []
    for impl in ("auto", "mma"):
        os.environ["ODP_ATTN_IMPL"] = impl
        name = "tcgen05" if attn.use_tc(S) else "mma.sync"
        f = _timeit(lambda: attn.fwd(qkv, GB, S, nh, nkv, cos, sin, o, lse), reps, flush)
        b = _timeit(lambda: attn.bwd(qkv, GB, S, nh, nkv, cos, sin, o, lse, do, delta, dqkv), reps, flush)
        check_errors()
        # algorithmic bytes: fwd reads q|k|v, writes o + lse; bwd reads q|k|v, o, do, lse, writes dq|dk|dv
        fb = qkv.numel() * 2 + o.numel() * 2 + lse.numel() * 4
        bb = qkv.numel() * 4 + o.numel() * 4 + lse.numel() * 4
        out.append({"kernel": f"attention_fwd[{name}]", "ms": round(f, 4), "GBps": round(fb / f / 1e6, 1),
                    "shape": [GB, S, nh, nkv]})
        out.append({"kernel": f"attention_bwd[{name}]", "ms": round(b, 4), "GBps": round(bb / b / 1e6, 1),
                    "shape": [GB, S, nh, nkv]})
    os.environ.pop("ODP_ATTN_IMPL", None)
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--paths", type=int, default=16)
    ap.add_argument("--batch", type=int, default=24)
    ap.add_argument("--seq", type=int, default=128)
    ap.add_argument("--heads", type=int, default=6)
    ap.add_argument("--kv-heads", type=int, default=6)
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    flush = torch.empty(64 * 1024 * 1024, device="cuda")
    cases = {"attention": lambda: bench_attention(args.paths * args.batch, args.seq, args.heads, args.kv_heads,
                                                  args.reps, flush)}
    for name, fn in cases.items():
        if args.only and args.only != name:
            continue
        for row in fn():
            print(json.dumps(row), flush=True)


if __name__ == "__main__":
    main()
