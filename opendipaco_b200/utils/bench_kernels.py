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


def _peaks() -> tuple[float, float, str]:
    """(bf16 TFLOP/s, HBM GB/s, label): the measured peaks written next to the repository
    (MEASURED_PEAKS.json: cuBLAS bf16 burst, STREAM-style copy) when present, else an
    earlier measurement on B200 (1590 TFLOP/s, 6650 GB/s)."""
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                        "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), float(d["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, 6650.0, "fallback"


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
    # causal attention FLOPs: forward Q K^T and P V over the lower triangle (S (S + 1) / 2
    # scores per head), backward five such products (S, dP, dV, dK, dQ)
    tri = GB * nh * S * (S + 1) / 2
    fwd_flops, bwd_flops = 2 * 2 * tri * D, 5 * 2 * tri * D
    tf, _, lab = _peaks()
    shp = attn.qkr_shape(GB, S, nh, nkv)
    qkr = torch.empty(shp, device=dev, dtype=torch.bfloat16) if shp else None
    variants = [("auto", qkr)] + ([("auto", None)] if qkr is not None else []) + [("mma", None)]
    for impl, q in variants:
        os.environ["ODP_ATTN_IMPL"] = impl
        name = {"tc": "tcgen05 one-tile", "flash": "tcgen05 flash", "mma": "mma.sync"}[attn.impl_for(S)]
        if attn.impl_for(S) == "flash":
            name += ", q|k rotated once" if q is not None else ", q|k rotated per tile"
        f = _timeit(lambda: attn.fwd(qkv, GB, S, nh, nkv, cos, sin, o, lse, qkr=q), reps, flush)
        b = _timeit(lambda: attn.bwd(qkv, GB, S, nh, nkv, cos, sin, o, lse, do, delta, dqkv, qkr=q), reps, flush)
        check_errors()
        # algorithmic bytes: fwd reads q|k|v, writes o + lse; bwd reads q|k|v, o, do, lse, writes dq|dk|dv
        fb = qkv.numel() * 2 + o.numel() * 2 + lse.numel() * 4
        bb = qkv.numel() * 4 + o.numel() * 4 + lse.numel() * 4
        out.append({"kernel": f"attention_fwd[{name}]", "ms": round(f, 4), "GBps": round(fb / f / 1e6, 1),
                    "TFLOPs": round(fwd_flops / f / 1e9, 1),
                    f"frac_of_{lab}_bf16_peak": round(fwd_flops / f / 1e9 / tf, 3), "shape": [GB, S, nh, nkv]})
        out.append({"kernel": f"attention_bwd[{name}]", "ms": round(b, 4), "GBps": round(bb / b / 1e6, 1),
                    "TFLOPs": round(bwd_flops / b / 1e9, 1),
                    f"frac_of_{lab}_bf16_peak": round(bwd_flops / b / 1e9 / tf, 3), "shape": [GB, S, nh, nkv]})
    os.environ.pop("ODP_ATTN_IMPL", None)
    return out


def bench_gemm(G: int, M: int, H: int, V: int, F: int, reps: int, flush) -> list[dict]:
    """The vocab-sized GEMMs of the LM head and the MLP GEMMs of one layer, grouped over
    G paths, with the epilogues the training step uses."""
    from ..ops._ext import check_errors
    from ..ops.gemm import gemm

    dev = torch.device("cuda")
    x = torch.randn(G, M, H, device=dev).to(torch.bfloat16)
    w = (torch.randn(G, V, H, device=dev) * 0.02).to(torch.bfloat16)
    logits = torch.empty(G, M, V, device=dev, dtype=torch.bfloat16)
    tiles_n = (V + 127) // 128
    part = torch.empty(G, M, 2 * tiles_n, 2, device=dev)
    dx = torch.empty(G, M, H, device=dev)
    dw = torch.empty(G, V, H, device=dev)
    wgu = (torch.randn(G, 2 * F, H, device=dev) * 0.02).to(torch.bfloat16)
    act = torch.empty(G, M, F, device=dev, dtype=torch.bfloat16)
    gu = torch.empty(G, M, 2 * F, device=dev, dtype=torch.bfloat16)
    wd = (torch.randn(G, H, F, device=dev) * 0.02).to(torch.bfloat16)
    y = torch.empty(G, M, H, device=dev, dtype=torch.bfloat16)
    cases = [
        ("logits x W^T (bf16 + row max/sumexp)", M, V, H,
         lambda: gemm(x, H, M * H, False, w, H, V * H, False, logits, V, M * V, M, V, H, G, "logits", part=part)),
        ("logits x W^T (plain bf16)", M, V, H,
         lambda: gemm(x, H, M * H, False, w, H, V * H, False, logits, V, M * V, M, V, H, G, "bf16")),
        ("dlogits x W (f32)", M, H, V,
         lambda: gemm(logits, V, M * V, False, w, H, V * H, True, dx, H, M * H, M, H, V, G, "f32")),
        ("dlogits^T x X (f32 dW)", V, H, M,
         lambda: gemm(logits, V, M * V, True, x, H, M * H, True, dw, H, V * H, V, H, M, G, "f32")),
        ("dlogits x W (f32, 192-wide tiles)", M, H, V,
         lambda: gemm(logits, V, M * V, False, w, H, V * H, True, dx, H, M * H, M, H, V, G, "f32", bn=192)),
        ("dlogits^T x X (f32 dW, 192-wide tiles)", V, H, M,
         lambda: gemm(logits, V, M * V, True, x, H, M * H, True, dw, H, V * H, V, H, M, G, "f32", bn=192)),
        ("X x Wgu^T (swiglu)", M, 2 * F, H,
         lambda: gemm(x, H, M * H, False, wgu, H, 2 * F * H, False, act, F, M * F, M, 2 * F, H, G, "swiglu",
                      aux=gu, ldx=2 * F, sx=M * 2 * F, f_half=F)),
        ("act x Wdown^T (bf16)", M, H, F,
         lambda: gemm(act, F, M * F, False, wd, F, H * F, False, y, H, M * H, M, H, F, G, "bf16")),
    ]
    # library reference points (cuBLAS through torch) for the same shapes, bf16 out
    cases += [
        ("[cuBLAS] logits x W^T", M, V, H, lambda: torch.bmm(x, w.transpose(1, 2), out=logits)),
        ("[cuBLAS] dlogits x W", M, H, V, lambda: torch.bmm(logits, w, out=y)),
    ]
    out = []
    for name, m, n, k, fn in cases:
        ms = _timeit(fn, reps, flush)
        check_errors()
        fl = 2.0 * G * m * n * k
        tf, _, lab = _peaks()
        out.append({"kernel": f"gemm {name}", "ms": round(ms, 4), "TFLOPs": round(fl / ms / 1e9, 1),
                    f"frac_of_{lab}_bf16_peak": round(fl / ms / 1e9 / tf, 3), "shape": [G, m, n, k]})
    return out


def bench_ce(G: int, M: int, V: int, reps: int, flush) -> list[dict]:
    """The cross-entropy kernels of the LM head on bf16 logits [G, M, V]."""
    from ..ops._ext import check_errors, err_word, ext

    dev = torch.device("cuda")
    logits = (torch.randn(G, M, V, device=dev) * 2).to(torch.bfloat16)
    labels = torch.randint(0, V, (G * M,), device=dev, dtype=torch.int32)
    tiles_n = (V + 127) // 128
    part = torch.randn(G, M, 2 * tiles_n, 2, device=dev)
    lse = torch.empty(G * M, device=dev)
    row_loss = torch.empty(G * M, device=dev)
    loss_sum = torch.empty(G, device=dev)
    inv = torch.ones(G, device=dev)
    x = ext()
    out = []
    cases = [
        ("ce_forward (finalize partials + group sums)",
         lambda: x.ce_forward(part, 2 * tiles_n, logits, V, M * V, labels, M, G, lse, row_loss, loss_sum, inv, None,
                              None),
         G * M * 2 * tiles_n * 8),
        ("ce_backward (in place, bf16)", lambda: x.ce_backward(logits, V, M * V, lse.zero_(), labels, inv, M, V, G),
         2 * logits.numel() * 2),
    ]
    if hasattr(x, "ce_fused"):
        cases.append(("ce_fused (loss + dlogits in place, bf16)",
                      lambda: x.ce_fused(logits, V, M * V, labels, M, V, G, lse, row_loss, loss_sum, inv, None, err_word(dev),
                                         None),
                      2 * logits.numel() * 2))
    for name, fn, nbytes in cases:
        ms = _timeit(fn, reps, flush)
        check_errors()
        _, bw, lab = _peaks()
        out.append({"kernel": name, "ms": round(ms, 4), "GBps": round(nbytes / ms / 1e6, 1),
                    f"frac_of_{lab}_hbm": round(nbytes / ms / 1e6 / bw, 3), "shape": [G, M, V]})
    return out


def bench_optim(G: int, H: int, V: int, F: int, layers: list[int], levels: list[int], reps: int, flush) -> list[dict]:
    """The inner optimizer on G paths of the DiPaCo layout (embedding, one region per
    level, head): plain AdamW, and the last step's AdamW that also accumulates the outer
    pseudo-gradient of every module key (paths on a level split over its experts)."""
    import numpy as np

    from ..ops._ext import check_errors, ext
    from ..train.fused import ACC_ENTRY, acc_region_table

    dev = torch.device("cuda")
    ru = lambda n: (n + 255) // 256 * 256  # noqa: E731
    per_layer = ru(3 * H * H) + ru(H * H) + ru(2 * F * H) + ru(H * F) + 2 * ru(H)
    sizes = [ru(V * H)] + [per_layer * n for n in layers] + [ru(H) + ru(V * H)]
    P = sum(sizes)
    w32, gr = torch.randn(G, P, device=dev), torch.randn(G, P, device=dev) * 1e-3
    m1, m2 = torch.zeros(G, P, device=dev), torch.zeros(G, P, device=dev)
    w16 = torch.empty(G, P, device=dev, dtype=torch.bfloat16)
    coef = torch.ones(G, device=dev)
    sched = torch.tensor([[1e-3, 1e-3 / 0.1, 0.3, 1.0]] * G, device=dev)
    # keys: the embedding and head shared by all G paths; level l's region split over
    # levels[l] experts (path g uses expert (g // stride) % levels[l])
    spans, o = [], 0
    for n in sizes:
        spans.append((o, o + n))
        o += n
    reg, ents, ctas = acc_region_table({sp: [0] * G for sp in spans})
    bufs, off = [], 0
    for r, n in enumerate(sizes):
        groups: dict[int, list[int]] = {}
        for g in range(G):
            if r in (0, len(sizes) - 1):
                expert = 0
            else:  # digit r - 1 of the mixed-radix path index g
                expert = (g // int(np.prod(levels[r:]))) % levels[r - 1]
            groups.setdefault(expert, []).append(g)
        for key in sorted(groups):
            d, gl = torch.zeros(n, device=dev), torch.randn(n, device=dev)
            bufs += [d, gl]
            for j, g in enumerate(groups[key]):
                ents.append((d.data_ptr(), gl.data_ptr(), g, int(j + 1 == len(groups[key])), 1.0 / G, 0))
        off += n
    rt = torch.from_numpy(reg.view(np.int64).copy()).to(dev)
    et = torch.from_numpy(np.array(ents, dtype=ACC_ENTRY).view(np.int64).copy()).to(dev)
    x = ext()
    nbytes = G * P * (4 * 4 + 3 * 4 + 2)  # p, g, m, v in; p, m, v, bf16 p out
    cases = [("adamw_step", lambda: x.adamw_step(w32, gr, m1, m2, w16, P, P, P, G, coef, sched, 0.9, 0.95, 1e-8, 0.1,
                                                 None, 0, 1, 1)),
             ("adamw_acc_step (+ outer pseudo-gradient)",
              lambda: x.adamw_acc_step(w32, gr, m1, m2, w16, ctas, P, P, coef, sched, 0.9, 0.95, 1e-8, 0.1, None, 0,
                                       1, 1, rt, len(sizes), et, True)),
             ("adamw_acc_step (no accumulation: the other inner steps)",
              lambda: x.adamw_acc_step(w32, gr, m1, m2, w16, ctas, P, P, coef, sched, 0.9, 0.95, 1e-8, 0.1, None, 0,
                                       1, 1, rt, len(sizes), et, False))]
    out = []
    _, bw, lab = _peaks()
    for name, fn in cases:
        ms = _timeit(fn, reps, flush)
        check_errors()
        out.append({"kernel": name, "ms": round(ms, 4), "GBps": round(nbytes / ms / 1e6, 1),
                    f"frac_of_{lab}_hbm": round(nbytes / ms / 1e6 / bw, 3), "shape": [G, P]})
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--paths", type=int, default=16)
    ap.add_argument("--batch", type=int, default=24)
    ap.add_argument("--seq", type=int, default=128)
    ap.add_argument("--heads", type=int, default=6)
    ap.add_argument("--kv-heads", type=int, default=6)
    ap.add_argument("--hidden", type=int, default=384)
    ap.add_argument("--ffn", type=int, default=1024)
    ap.add_argument("--vocab", type=int, default=32000)
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    flush = torch.empty(64 * 1024 * 1024, device="cuda")
    cases = {"attention": lambda: bench_attention(args.paths * args.batch, args.seq, args.heads, args.kv_heads,
                                                  args.reps, flush),
             "gemm": lambda: bench_gemm(args.paths, args.batch * args.seq, args.hidden, args.vocab, args.ffn,
                                        args.reps, flush),
             "ce": lambda: bench_ce(args.paths, args.batch * args.seq, args.vocab, args.reps, flush),
             "optim": lambda: bench_optim(args.paths, args.hidden, args.vocab, args.ffn, [2, 2], [4, 4], args.reps,
                                          flush)}
    for name, fn in cases.items():
        if args.only and args.only != name:
            continue
        for row in fn():
            print(json.dumps(row), flush=True)


if __name__ == "__main__":
    main()
