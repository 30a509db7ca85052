"""m3r_match_nn_static: the matcher arg-max for callers that cannot allocate device memory
(a real-time loop that cannot absorb cudaMalloc's device synchronisation, or a framework
that owns all GPU memory in its own pool).  The entry point itself allocates nothing:
its temporaries live in a static device array inside the library.  This test allocates
the caller's input and output buffers (with torch, standing in for such a caller's own
pool) and checks the results against m3r_match_nn, bit for bit, on two calls in a row
with different sizes -- the second call reuses the array the first one left behind.

This file is named so that pytest collects it last."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _reference(lib, a, b):
    from mast3r_runtime_b200 import _lib

    n1, d = a.shape
    n2 = b.shape[0]
    nn12 = np.zeros(n1, np.int32)
    nn21 = np.zeros(n2, np.int32)
    best = np.zeros(n1, np.float32)
    ms = ctypes.c_float(0)
    _lib.check(lib.m3r_match_nn(0, _lib.ptr(a), _lib.ptr(b), n1, n2, d, _lib.ptr(nn12), _lib.ptr(nn21),
                                _lib.ptr(best), ctypes.byref(ms)))
    return nn12, nn21, best


def test_match_nn_static_equals_match_nn_on_two_calls():
    import torch

    from mast3r_runtime_b200 import _lib

    lib = _lib.load()
    for n1, n2, d, seed in ((3000, 2500, 24, 1), (1200, 4000, 64, 2)):
        rng = np.random.default_rng(seed)
        a = rng.standard_normal((n1, d)).astype(np.float32)
        b = rng.standard_normal((n2, d)).astype(np.float32)
        b[: n2 // 5] = a[rng.integers(0, n1, n2 // 5)]  # exact copies: tied similarities
        want12, want21, wantb = _reference(lib, a, b)

        dev = torch.device("cuda", 0)
        ta = torch.from_numpy(a).to(dev)
        tb = torch.from_numpy(b).to(dev)
        o12 = torch.full((n1,), -1, dtype=torch.int32, device=dev)
        o21 = torch.full((n2,), -1, dtype=torch.int32, device=dev)
        ob = torch.zeros(n1, dtype=torch.float32, device=dev)
        stream = torch.cuda.current_stream(dev).cuda_stream
        torch.cuda.synchronize(dev)
        free_before = torch.cuda.mem_get_info(dev)[0]
        rc = lib.m3r_match_nn_static(0, ta.data_ptr(), tb.data_ptr(), n1, n2, d, o12.data_ptr(), o21.data_ptr(),
                                     ob.data_ptr(), stream)
        _lib.check(rc)
        torch.cuda.synchronize(dev)
        if seed > 1:
            # past its first (set-up) call the entry point allocates no device memory:
            # the device's free memory is unchanged (allocations come in >= 2 MiB pages)
            assert torch.cuda.mem_get_info(dev)[0] == free_before
        np.testing.assert_array_equal(o12.cpu().numpy(), want12)
        np.testing.assert_array_equal(o21.cpu().numpy(), want21)
        assert ob.cpu().numpy().tobytes() == wantb.tobytes()


def test_match_nn_static_rejects_sizes_beyond_its_array():
    from mast3r_runtime_b200 import _lib

    lib = _lib.load()
    rc = lib.m3r_match_nn_static(0, 16, 16, 16385, 10, 24, 16, 16, None, None)  # never dereferenced
    assert rc == -1
    assert b"static scratch limit" in lib.m3r_global_error()
    rc = lib.m3r_match_nn_static(0, 16, 16, 10, 10, 65, 16, 16, None, None)
    assert rc == -1
