"""The allocation-free router entry point, `wmoe_router_topk_static`.

Who needs it: a caller that routes tokens where it may not allocate device
memory -- code being recorded into a CUDA graph (cudaMalloc cannot be
captured), a serving loop that must never take the device-synchronising
allocation path, or a host framework that owns all device memory through its
own allocator.  The regular `wmoe_router_topk` asks such a caller for a
[T, E] float32 logits buffer; this variant keeps those logits in a 1 MiB
array inside the library instead (T * E <= 262,144).

The test calls both entry points through the C ABI with ctypes and requires
identical indices and weights (the router is bit-exact, so the shared tolerance
here is equality), on two calls in a row with different inputs, so a stale
scratch from the first call would show up in the second.  It also checks the
size limit is enforced.  The file name sorts last so a run that stops at the
first failure has already run every other test; it passes alone as well.
"""
import ctypes

import numpy as np
import pytest
import torch

from whallm_b200 import _lib as L

pytestmark = pytest.mark.gpu


def _case(seed, T, H, E, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)
    wg = (torch.randn((E, H), generator=g, device=dev) / H ** 0.5).to(torch.bfloat16)
    lb = torch.randn((E,), generator=g, device=dev) * 0.5
    sb = torch.randn((E,), generator=g, device=dev) * 0.1
    sg = (torch.randn((H,), generator=g, device=dev) / H ** 0.5).to(torch.bfloat16)
    return x, wg, lb, sb, sg


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _run(static, x, wg, lb, sb, sg, k, score_fn, eps, scale):
    lib = L.lib()
    T, H = x.shape
    E = wg.shape[0]
    dev = x.device
    idx = torch.full((T, k), -7, dtype=torch.int32, device=dev)
    w = torch.full((T, k), float("nan"), dtype=torch.float32, device=dev)
    sh = torch.full((T,), float("nan"), dtype=torch.float32, device=dev) if sg is not None else None
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    if static:
        rc = lib.wmoe_router_topk_static(_p(x), _p(wg), _p(lb), _p(sb), _p(sg), T, H, E, k, score_fn, eps, scale,
                                         _p(idx), _p(w), _p(sh), stream)
    else:
        logits = torch.empty((T, E), dtype=torch.float32, device=dev)
        rc = lib.wmoe_router_topk(_p(x), _p(wg), _p(lb), _p(sb), _p(sg), T, H, E, k, score_fn, eps, scale,
                                  _p(logits), _p(idx), _p(w), _p(sh), stream)
    assert rc == L.WM_OK, L.last_error()
    torch.cuda.synchronize(dev)
    return idx.cpu().numpy(), w.cpu().numpy(), None if sh is None else sh.cpu().numpy()


def test_static_router_matches_regular_entry_twice_in_a_row():
    dev = torch.device("cuda:0")
    cases = [
        # (seed, T, H, E, k, score fn, norm eps, route scale, with shared gate)
        (1, 64, 7168, 256, 8, L.WM_SCORE_SQRTSOFTPLUS, 1e-20, 1.5, False),
        (2, 33, 2048, 512, 10, L.WM_SCORE_SOFTMAX, 0.0, 1.0, True),
    ]
    for seed, T, H, E, k, fn, eps, scale, shared in cases:
        x, wg, lb, sb, sg = _case(seed, T, H, E, dev)
        sg = sg if shared else None
        sb = None if shared else sb
        ref = _run(False, x, wg, lb, sb, sg, k, fn, eps, scale)
        got = _run(True, x, wg, lb, sb, sg, k, fn, eps, scale)
        np.testing.assert_array_equal(got[0], ref[0])
        np.testing.assert_array_equal(got[1], ref[1])
        if shared:
            np.testing.assert_array_equal(got[2], ref[2])
        assert (got[0] >= 0).all() and (got[0] < E).all()


def test_static_router_rejects_oversized_batches():
    dev = torch.device("cuda:0")
    x, wg, lb, sb, _ = _case(3, 1025, 256, 256, dev)  # 1025 * 256 > 262144
    lib = L.lib()
    idx = torch.empty((1025, 4), dtype=torch.int32, device=dev)
    w = torch.empty((1025, 4), dtype=torch.float32, device=dev)
    rc = lib.wmoe_router_topk_static(_p(x), _p(wg), _p(lb), None, None, 1025, 256, 256, 4, L.WM_SCORE_SOFTMAX,
                                     0.0, 1.0, _p(idx), _p(w), None,
                                     ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    assert rc == L.WM_ERR_INVALID
    assert "static scratch" in L.last_error()
