"""Failure detection on the device without a GPU fault: a cross-GPU wait that runs out.

The outer-step APPLY kernel and the data-parallel barrier wait for flags that other GPUs
write. Here, on one GPU, each is launched as a member of a two-rank group whose second
rank never exists: its flag lives in an ordinary local buffer that nothing writes. With
the wait bound shortened to 20 ms, the kernel must give up, record ERR_TIMEOUT_PEER in
the error word and return; the host must raise ``KernelTimeout``; and the context must
stay usable, so the next launch (a healthy one-rank APPLY) computes the right answer.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"
WAIT_NS = 20_000_000  # 20 ms


@pytest.fixture
def short_wait():
    from opendipaco_b200.ops._ext import ext

    old = ext().set_peer_wait_ns(WAIT_NS)
    yield
    ext().set_peer_wait_ns(old)


def _ptrs(*ts):
    return torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device=DEV)


def _one_key(n):
    from opendipaco_b200.parallel.backend.nvlink import NVKEY

    rec = np.zeros(1, dtype=NVKEY)
    rec["off"], rec["s0"], rec["s1"], rec["chunk0"], rec["nsh"] = 0, 0, n, 0, 1
    rec["sh"][0, 0] = 0
    rec["scale"], rec["inv_den"], rec["quant"] = 1.0, 1.0, 0
    return torch.from_numpy(rec.view(np.int64).copy()).to(DEV)


def test_outer_apply_peer_wait_times_out_and_context_survives(short_wait):
    from opendipaco_b200.ops._ext import KernelTimeout, check_errors, err_word, ext

    n = 4096
    keys = _one_key(n)
    delta = torch.ones(n, device=DEV)
    glob = torch.zeros(n, device=DEV)
    mom = torch.zeros(n, device=DEV)
    sq = torch.zeros(1, device=DEV)
    err = err_word(torch.device(DEV))
    check_errors()
    # rank 0 of a 2-rank group; "rank 1"'s pad is a local buffer nobody publishes into
    pad0 = torch.zeros(4, dtype=torch.int32, device=DEV)
    pad1 = torch.zeros(4, dtype=torch.int32, device=DEV)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    ext().outer_nvlink_apply(keys, 1, 1, _ptrs(delta, delta), _ptrs(glob, glob), _ptrs(pad0, pad1), mom, 0, 2, 1,
                             0.5, 0.9, True, True, sq, err, None, None, 0, None)
    ev1.record()
    torch.cuda.synchronize()
    waited_ms = ev0.elapsed_time(ev1)
    assert int(err.item()) == 5  # ERR_TIMEOUT_PEER
    with pytest.raises(KernelTimeout, match="peer flag never arrived"):
        check_errors()
    assert int(err.item()) == 0  # check_errors clears the word it reported
    # the wait gave up after the bound (not the 2 s default) and nothing was updated
    assert WAIT_NS / 1e6 <= waited_ms < 1000.0, waited_ms
    assert torch.equal(glob, torch.zeros(n, device=DEV)) and torch.equal(mom, torch.zeros(n, device=DEV))
    # the context is intact: a one-rank APPLY on the same buffers runs to completion
    ext().outer_nvlink_apply(keys, 1, 1, _ptrs(delta), _ptrs(glob), _ptrs(pad0), mom, 0, 1, 2,
                             0.5, 0.9, True, True, sq, err, None, None, 0, None)
    torch.cuda.synchronize()
    check_errors()
    # first outer step, Nesterov: b = d, update = d + m * d, glob = -lr * 1.9 * d
    assert torch.allclose(glob, torch.full((n,), -0.5 * 1.9, device=DEV))
    assert torch.allclose(mom, torch.ones(n, device=DEV))


def test_data_parallel_barrier_times_out(short_wait):
    from opendipaco_b200.ops._ext import KernelTimeout, check_errors, err_word, ext

    # pointer table int64 [rows][8]: row 5 (PAD) holds each member's flag pad
    tab = torch.zeros(12, 8, dtype=torch.int64, device=DEV)
    pad0 = torch.zeros(8, dtype=torch.int32, device=DEV)
    pad1 = torch.zeros(8, dtype=torch.int32, device=DEV)
    tab[5, 0], tab[5, 1] = pad0.data_ptr(), pad1.data_ptr()
    counter = torch.zeros(1, dtype=torch.int32, device=DEV)
    err = err_word(torch.device(DEV))
    check_errors()
    ext().dp_barrier(tab, counter, 0, 2, err)
    torch.cuda.synchronize()
    with pytest.raises(KernelTimeout):
        check_errors()
    # this member did publish its arrival to both pads before giving up on member 1
    assert int(pad0[0].item()) == 1 and int(pad1[0].item()) == 1
    # a one-member group passes its barrier on the same context
    ext().dp_barrier(tab, counter, 0, 1, err)
    torch.cuda.synchronize()
    check_errors()
    assert int(counter.item()) == 2
