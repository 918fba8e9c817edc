"""The outer step's fused pieces on one GPU: the last inner step's AdamW that also
accumulates the outer pseudo-gradient (``adamw_acc_step``), checked bit for bit against
plain AdamW followed by the separate accumulation pass; the non-finite guard of the
outer step; and the vectorised modes (ACC + APPLY == OUTER) of ``outer_step``."""

import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _sched(G, lr=1e-3, t=3, b1=0.9, b2=0.95, active=None):
    rows = []
    for g in range(G):
        act = 1.0 if active is None or active[g] else 0.0
        rows.append([lr, lr / (1 - b1 ** t), math.sqrt(1 - b2 ** t), act])
    return torch.tensor(rows, device=DEV, dtype=torch.float32)


def test_adamw_acc_equals_adamw_then_accumulate_bitwise():
    from opendipaco_b200.ops._ext import ext
    from opendipaco_b200.ops.outer import MODE_ACC, OuterPlan, Segment
    from opendipaco_b200.train.fused import ACC_ENTRY, acc_region_table

    torch.manual_seed(0)
    G, P = 4, 4096 * 3
    # path layout: region A [0, 4096) shared by all four paths (key "a"), region B
    # [4096, 8192) split over two keys (paths 0, 2 -> "b0"; 1, 3 -> "b1"), region C
    # [8192, 12288) private to each path ("c0".."c3")
    regions = {"A": (0, 4096), "B": (4096, 8192), "C": (8192, 12288)}
    keys_of = {g: ["a", "b0" if g % 2 == 0 else "b1", f"c{g}"] for g in range(G)}
    region_of = {"a": "A", "b0": "B", "b1": "B", **{f"c{g}": "C" for g in range(G)}}
    weights = {("a", 0): 0.1, ("a", 1): 0.2, ("a", 2): 0.3, ("a", 3): 0.4, ("b0", 0): 0.5, ("b0", 2): 0.5,
               ("b1", 1): 0.25, ("b1", 3): 0.0}
    active = [True, True, True, False]
    W = torch.randn(G, P, device=DEV)
    GR = torch.randn(G, P, device=DEV)
    M1 = torch.randn(G, P, device=DEV) * 0.01
    M2 = torch.rand(G, P, device=DEV) * 0.01
    coef = torch.tensor([1.0, 0.5, 0.25, 1.0], device=DEV)
    sched = _sched(G, active=active)
    glob = {k: torch.randn(4096, device=DEV) for k in ("a", "b0", "b1")}
    glob.update({f"c{g}": torch.zeros(4096, device=DEV) for g in range(G)})

    def run(fused, accumulate=True):
        w32, m1, m2 = W.clone(), M1.clone(), M2.clone()
        w16 = torch.zeros(G, P, device=DEV, dtype=torch.bfloat16)  # the inactive path's copy is never written
        gl = {k: v.clone() for k, v in glob.items()}
        delta = {k: torch.full((4096,), float("nan"), device=DEV) for k in ("a", "b0", "b1")}
        if fused:
            order = {k: i for i, k in enumerate(["a", "b0", "b1"] + [f"c{g}" for g in range(G)])}
            lists = {r: [] for r in regions}
            for g in range(G):
                for k in keys_of[g]:
                    lists[region_of[k]].append((order[k], g, k))
            reg, ents, ctas = acc_region_table({regions[r]: lists[r] for r in regions})
            for r in sorted(regions, key=lambda r: regions[r][0]):
                lst = sorted(lists[r])
                for i, (_, g, k) in enumerate(lst):
                    last = i + 1 == len(lst) or lst[i + 1][2] != k
                    d = 0 if k.startswith("c") else delta[k].data_ptr()
                    ents.append((d, gl[k].data_ptr(), g, int(last), weights.get((k, g), 0.0) if active[g] else 0.0, 0))
            rt = torch.from_numpy(reg.view(np.int64).copy()).to(DEV)
            et = torch.from_numpy(np.array(ents, dtype=ACC_ENTRY).view(np.int64).copy()).to(DEV)
            ext().adamw_acc_step(w32, GR, m1, m2, w16, ctas, P, P, coef, sched, 0.9, 0.95, 1e-8, 0.1, None, 0, 1,
                                 1, rt, 3, et, accumulate)
        else:
            ext().adamw_step(w32, GR, m1, m2, w16, P, P, P, G, coef, sched, 0.9, 0.95, 1e-8, 0.1, None, 0, 1, 1)
            if not accumulate:
                torch.cuda.synchronize()
                return w32, w16, m1, m2, gl, delta
            segs = []
            for k in ("a", "b0", "b1"):
                users = [g for g in range(G) if k in keys_of[g]]
                a, b = regions[region_of[k]]
                segs.append(Segment(k, gl[k], None, [w32[g, a:b] for g in users], [None] * len(users),
                                    [weights.get((k, g), 0.0) if active[g] else 0.0 for g in users], MODE_ACC,
                                    delta=delta[k]))
            OuterPlan(segs, DEV).run(0.0, 0.0, False, False)
            for g in range(G):
                a, b = regions["C"]
                gl[f"c{g}"].copy_(w32[g, a:b])
        torch.cuda.synchronize()
        return w32, w16, m1, m2, gl, delta

    ref, got = run(False), run(True)
    for x, y in zip(ref[:4], got[:4]):
        assert torch.equal(x, y)
    for k in glob:
        assert torch.equal(ref[4][k], got[4][k]), k
    for k in ("a", "b0", "b1"):
        assert torch.equal(ref[5][k], got[5][k]), k
    # the inactive path's weights are untouched and its pseudo-gradient weight is zero
    assert torch.equal(got[0][3], W[3])
    # the other inner steps: the same AdamW, and the outer buffers are left alone
    plain, region = run(False, accumulate=False), run(True, accumulate=False)
    for x, y in zip(plain[:4], region[:4]):
        assert torch.equal(x, y)
    for k in glob:
        assert torch.equal(region[4][k], glob[k])
    assert all(torch.isnan(region[5][k]).all() for k in ("a", "b0", "b1"))


def test_outer_guard_skips_non_finite_elements():
    from opendipaco_b200.ops.outer import OuterPlan, Segment

    n = 8192
    glob = torch.randn(n, device=DEV)
    mom = torch.randn(n, device=DEV) * 0.1
    locs = [glob + 0.01 * torch.randn(n, device=DEV) for _ in range(2)]
    locs[1][100] = float("nan")
    locs[0][5000:5004] = float("inf")
    l16 = [torch.empty(n, device=DEV, dtype=torch.bfloat16) for _ in range(2)]
    w = [0.5, 0.5]
    g0, m0 = glob.clone(), mom.clone()
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    plan = OuterPlan([Segment("k", glob, mom, locs, l16, w, scale=1.0)], DEV)
    # expected with PyTorch, elements with a non-finite pseudo-gradient held back
    acc = 0.5 * (g0 - locs[0]) + 0.5 * (g0 - locs[1])
    bad = ~torch.isfinite(acc)
    b = torch.where(bad, m0, 0.9 * m0 + acc)
    upd = acc + 0.9 * b
    new = torch.where(bad, g0, g0 - 0.7 * upd)
    plan.run(0.7, 0.9, True, first=False, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == int(bad.sum().item()) == 5
    assert torch.equal(glob[bad], g0[bad]) and torch.equal(mom[bad], m0[bad])
    torch.testing.assert_close(glob, new, rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(mom, b, rtol=1e-6, atol=1e-6)
    for l, h in zip(locs, l16):
        assert torch.equal(l, glob)  # diverged copies are reset to the global
        assert torch.equal(h, glob.to(torch.bfloat16))
    assert torch.isfinite(plan.sq_part).all()


def test_acc_then_apply_equals_one_pass_outer_step():
    from opendipaco_b200.ops.outer import MODE_ACC, MODE_APPLY, OuterPlan, Segment

    torch.manual_seed(1)
    n = 3 * 4096 + 512
    base = torch.randn(n, device=DEV)

    def setup():
        glob, mom = base.clone(), torch.full((n,), 0.05, device=DEV)
        locs = [base + 0.01 * torch.randn(n, device=DEV, generator=torch.Generator(DEV).manual_seed(j))
                for j in range(5)]
        return glob, mom, locs, [torch.empty(n, device=DEV, dtype=torch.bfloat16) for _ in range(5)]

    w = [0.1, 0.2, 0.3, 0.15, 0.25]
    g1, m1, l1, h1 = setup()
    OuterPlan([Segment("k", g1, m1, l1, h1, w, scale=2.0, inv_den=0.5)], DEV).run(0.7, 0.9, True, False)
    g2, m2, l2, h2 = setup()
    delta = torch.empty(n, device=DEV)
    OuterPlan([Segment("k", g2, m2, l2, h2, w, MODE_ACC, 2.0, 0.5, delta)], DEV).run(0.0, 0.0, False, False)
    OuterPlan([Segment("k", g2, m2, l2, h2, w, MODE_APPLY, 2.0, 0.5, delta)], DEV).run(0.7, 0.9, True, False)
    torch.cuda.synchronize()
    assert torch.equal(g1, g2) and torch.equal(m1, m2)
    for a, b in zip(l1 + h1, l2 + h2):
        assert torch.equal(a, b)
