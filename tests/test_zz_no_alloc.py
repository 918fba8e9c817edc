"""The allocation-free clip-coefficient entry point, called through its exported C symbol.

``odp_grad_clip_coef_noalloc`` serves callers that cannot allocate GPU memory (a process
that reserved all device memory for its own pool, a step loop that allows no allocation,
C code without torch's allocator): it keeps its scratch in a fixed static device array.
These tests load the symbol with ctypes, as such a caller would, and check it against the
library's usual entry point (``ops.adam.clip_coef``, which takes a scratch tensor) and an
fp32 PyTorch reference, on calls made back to back so that the second call sees the
scratch the first one left behind.

The file name sorts last so that a run stopping at its first failure has already run
every other test.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_GROUPS = 64
MAX_BLOCKS = 4096
ELEMS_PER_BLOCK = 1 << 16


def _fn():
    from opendipaco_b200.ops._ext import ext

    lib = ctypes.CDLL(ext().__file__)
    f = lib.odp_grad_clip_coef_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_longlong, ctypes.c_int, ctypes.c_float,
                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    return f


def _call(f, g, P, stride, G, max_norm, coef, norm):
    stream = torch.cuda.current_stream().cuda_stream
    return f(g.data_ptr(), P, stride, G, max_norm, coef.data_ptr(), norm.data_ptr() if norm is not None else None,
             stream)


def _reference(g, P, G, max_norm):
    norm = torch.stack([g[i, :P].double().pow(2).sum().sqrt() for i in range(G)]).float()
    coef = torch.clamp(max_norm / (norm + 1e-6), max=1.0) if max_norm > 0 else torch.ones_like(norm)
    return norm, coef


def test_matches_existing_entry_point_on_back_to_back_calls():
    from opendipaco_b200.ops.adam import clip_coef

    f = _fn()
    dev = torch.device("cuda:0")
    torch.manual_seed(0)
    # first call: many paths, several blocks each, a ragged tail; second call: fewer,
    # shorter paths, so stale partials of the first call sit in the shared scratch
    for G, P, stride, scale, max_norm in ((12, 3 * ELEMS_PER_BLOCK + 1234, 3 * ELEMS_PER_BLOCK + 1236, 0.02, 1.0),
                                          (5, 70001, 70004, 3.0, 0.5)):
        g = torch.randn(G, stride, device=dev) * scale
        coef = torch.full((G,), -1.0, device=dev)
        norm = torch.full((G,), -1.0, device=dev)
        assert _call(f, g, P, stride, G, max_norm, coef, norm) == 0
        norm_ref = torch.empty(G, device=dev)
        coef_ref = clip_coef(g, P, stride, G, max_norm, norm_out=norm_ref)
        torch.cuda.synchronize()
        # same partial layout and the same fixed-order tree: bit-identical results
        assert torch.equal(coef, coef_ref)
        assert torch.equal(norm, norm_ref)
        n32, c32 = _reference(g, P, G, max_norm)
        torch.testing.assert_close(norm, n32, rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(coef, c32, rtol=1e-4, atol=1e-5)


def test_rejects_sizes_beyond_the_static_scratch():
    f = _fn()
    dev = torch.device("cuda:0")
    g = torch.zeros(MAX_GROUPS + 1, 64, device=dev)
    coef = torch.zeros(MAX_GROUPS + 1, device=dev)
    assert _call(f, g, 64, 64, MAX_GROUPS + 1, 1.0, coef, None) == -1
    too_long = MAX_BLOCKS * ELEMS_PER_BLOCK + 4
    # only the sizes are checked before rejection, so a small buffer is enough here
    assert f(g.data_ptr(), too_long, too_long, 1, 1.0, coef.data_ptr(), None,
             torch.cuda.current_stream().cuda_stream) == -2
    assert _call(f, g, 60, 62, 2, 1.0, coef, None) == -3          # stride not a multiple of 4
    host = torch.zeros(4, 64)
    assert f(host.data_ptr(), 64, 64, 1, 1.0, coef.data_ptr(), None,
             torch.cuda.current_stream().cuda_stream) == -5      # not device memory
    # a rejected call launched nothing and left the device usable
    ok = torch.zeros(2, device=dev)
    assert _call(f, torch.ones(2, 64, device=dev), 64, 64, 2, 0.0, ok, None) == 0
    torch.cuda.synchronize()
    assert torch.equal(ok, torch.ones(2, device=dev))
