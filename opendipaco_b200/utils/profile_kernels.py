"""Launch each kernel family once at a profiling-sized shape (for a kernel profiler).

    python -m opendipaco_b200.utils.profile_kernels [--only adamw,outer,...]

Every case first runs its kernels twice untimed (warm-up: attributes, caches), then once
more -- so a profiler can skip the warm-up launches and capture exactly one launch of
each kernel. Shapes are chosen so that each kernel's working set is larger than the 126
MB L2 (its DRAM figures mean something) but the whole process stays within a few GB:

* adamw:     region AdamW (+ pseudo-gradient) over 2 paths of the 16-path layout (~1.1 GB)
* adam8bit:  blockwise 8-bit Adam over the same 2 x 31.7 M elements
* outer:     the one-GPU outer step (APPLY + write-back) over 2 x 12.3 M elements
* norm:      RMSNorm forward / backward, 2 x 3072 rows of 384
* embedding: the sorted deterministic embedding backward, 2 x 3072 tokens, vocab 32000
* attention: tcgen05 flash forward / backward (q|k rotated once), 4 x 1024 tokens, 32 / 8 heads
* ce:        one-pass cross-entropy, 2 x 3072 rows of 32000
* routing:   bag-of-tokens featurizer, tensor-core k-means assignment and the ordered
             centroid sums, 20000 documents x 256 features, 16 centroids
* codec:     int4 quantisation with error feedback, 32 M elements
"""

from __future__ import annotations

import argparse
import math

import torch


def _thrice(fn) -> None:
    fn()
    fn()
    torch.cuda.synchronize()
    fn()
    torch.cuda.synchronize()


def case_adamw() -> None:
    from .bench_kernels import bench_optim

    flush = torch.empty(1, device="cuda")
    bench_optim(2, 384, 32000, 1024, [2, 2], [4, 4], 1, flush)


def case_adam8bit() -> None:
    from ..ops._ext import ext

    G, P = 2, 31_658_496
    nb = P // 256
    w = torch.randn(G * P, device="cuda") * 0.02
    g = torch.randn(G * P, device="cuda") * 1e-3
    w16 = torch.empty(G * P, device="cuda", dtype=torch.bfloat16)
    mq = torch.zeros(G * nb, 256, device="cuda", dtype=torch.int8)
    vq = torch.zeros(G * nb, 256, device="cuda", dtype=torch.uint8)
    mabs, vlo, vsc = (torch.zeros(G * nb, device="cuda") for _ in range(3))
    coef = torch.ones(G, device="cuda")
    sched = torch.tensor([[1e-3, 1e-2, 0.2236, 1.0]] * G, device="cuda")  # lr, lr / bc1, sqrt(bc2), active
    _thrice(lambda: ext().adam8bit_step(w, g, mq, mabs, vq, vlo, vsc, coef, sched, 0.9, 0.95, 1e-8, 0.1, False, w16,
                                        nb))


def case_outer() -> None:
    from ..ops.outer import MODE_APPLY, OuterPlan, Segment

    n = 12_288_000
    glob = torch.randn(n, device="cuda")
    mom = torch.zeros(n, device="cuda")
    delta = torch.randn(n, device="cuda") * 1e-3
    locs = [glob.clone() for _ in range(2)]
    l16 = [torch.empty(n, device="cuda", dtype=torch.bfloat16) for _ in range(2)]
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    plan = OuterPlan([Segment("embed", glob, mom, locs, l16, [0.5, 0.5], MODE_APPLY, 1.0, 1.0, delta)], "cuda")
    _thrice(lambda: plan.run(0.7, 0.9, True, False, status))


def case_norm() -> None:
    from ..ops._ext import ext

    G, M, H = 2, 3072, 384
    x = torch.randn(G, M, H, device="cuda")
    w = torch.rand(G, H, device="cuda") + 0.5
    y = torch.empty(G, M, H, device="cuda", dtype=torch.bfloat16)
    rstd = torch.empty(G, M, device="cuda")
    dy = torch.randn(G, M, H, device="cuda")
    dx = torch.empty_like(x)
    dx16 = torch.empty(G, M, H, device="cuda", dtype=torch.bfloat16)
    dw = torch.empty(G, H, device="cuda")
    work = torch.empty(G * ((M + 7) // 8) * H, device="cuda")
    _thrice(lambda: ext().rmsnorm_fwd(x, M * H, w, H, y, M * H, rstd, M, H, G, 1e-5))
    _thrice(lambda: ext().rmsnorm_bwd(x, M * H, w, H, rstd, dy, M * H, None, dx, M * H, dx16, dw, H, work, M, H, G,
                                      0.0))


def case_embedding() -> None:
    from ..ops._ext import ext

    G, M, H, V = 2, 3072, 384, 32000
    ids = torch.randint(0, V, (G, M), device="cuda", dtype=torch.int32)
    dx = torch.randn(G, M, H, device="cuda")
    dE = torch.zeros(G, V * H, device="cuda")
    keys = torch.empty(G, M, dtype=torch.int32, device="cuda")
    rows = torch.zeros(G, V, dtype=torch.uint8, device="cuda")
    sq = torch.empty(G, M, device="cuda")
    _thrice(lambda: ext().embedding_bwd_sorted(ids, dx, M * H, dE, V * H, M, H, G, V, keys, rows, sq))


def case_attention() -> None:
    from ..models.llama import rope_cos_sin
    from ..ops import attention as attn

    GB, S, nh, nkv = 4, 1024, 32, 8
    cos, sin = rope_cos_sin(64, 10000.0, S, torch.device("cuda"))
    qkv = (torch.randn(GB, S, (nh + 2 * nkv) * 64, device="cuda")).to(torch.bfloat16)
    o = torch.empty(GB, S, nh * 64, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(GB, nh, S, device="cuda")
    do = torch.randn_like(o)
    delta = torch.empty(GB, nh, S, device="cuda")
    dqkv = torch.empty_like(qkv)
    qkr = torch.empty(attn.qkr_shape(GB, S, nh, nkv), device="cuda", dtype=torch.bfloat16)
    _thrice(lambda: attn.fwd(qkv, GB, S, nh, nkv, cos, sin, o, lse, qkr=qkr))
    _thrice(lambda: attn.bwd(qkv, GB, S, nh, nkv, cos, sin, o, lse, do, delta, dqkv, qkr=qkr))


def case_ce() -> None:
    from ..ops._ext import err_word, ext

    G, M, V = 2, 3072, 32000
    logits = (torch.randn(G, M, V, device="cuda") * 2).to(torch.bfloat16)
    labels = torch.randint(0, V, (G * M,), device="cuda", dtype=torch.int32)
    lse, row, loss_sum, inv = (torch.empty(G * M, device="cuda"), torch.empty(G * M, device="cuda"),
                               torch.empty(G, device="cuda"), torch.ones(G, device="cuda"))
    err = err_word(torch.device("cuda"))
    _thrice(lambda: ext().ce_fused(logits, V, M * V, labels, M, V, G, lse, row, loss_sum, inv, None, err, None))


def case_routing() -> None:
    from ..ops import routing as K

    N, D, V, K_ = 20000, 256, 32000, 16
    g = torch.Generator().manual_seed(0)
    docs = [torch.randint(0, V, (32,), generator=g) for _ in range(N)]
    proj = torch.randn(V, D, device="cuda") / math.sqrt(D)
    x = torch.randn(N, D, device="cuda")
    c = torch.randn(K_, D, device="cuda")
    _thrice(lambda: K.bag_of_tokens(docs, proj, V))
    _thrice(lambda: K.kmeans_assign(x, c, 2))
    idx = K.kmeans_assign(x, c, 1)
    _thrice(lambda: K.cluster_sums(x, idx, K_))


def case_codec() -> None:
    from ..ops import codec

    x = torch.randn(32 * 1024 * 1024, device="cuda")
    _thrice(lambda: codec.quant_int4(x))


CASES = {"adamw": case_adamw, "adam8bit": case_adam8bit, "outer": case_outer, "norm": case_norm, "embedding": case_embedding,
         "attention": case_attention, "ce": case_ce, "routing": case_routing, "codec": case_codec}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default=None, help="comma-separated cases (default: all)")
    args = ap.parse_args()
    names = args.only.split(",") if args.only else list(CASES)
    for name in names:
        CASES[name]()
        torch.cuda.synchronize()
        print(f"{name}: ok", flush=True)
    from ..ops._ext import check_errors

    check_errors()


if __name__ == "__main__":
    main()
