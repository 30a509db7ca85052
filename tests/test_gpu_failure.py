"""Failure detection on the GPU without a fault: every tcgen05 kernel waits on its
pipeline barriers with a bounded wait (a limit in ns, m3r_set_wait_timeout).  The
self-test kernel waits on a barrier that nothing signals; the wait must give up after
its limit, record its code, and the call must report M3R_ERR_TIMEOUT -- after which the
same process keeps using the GPU normally."""

from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest

from conftest import from16, rel_l2, round16, to16

pytestmark = pytest.mark.gpu

M3R_ERR_TIMEOUT = -5
KDEV_TIMEOUT_MMA = 2


@pytest.fixture(scope="module")
def lib():
    from mast3r_runtime_b200 import _lib

    return _lib.load()


def _attention_ok(lib):
    from mast3r_runtime_b200 import _lib

    rng = np.random.default_rng(5)
    s, h, n = 2, 2, 200
    q, k, v = (round16(rng.standard_normal((s, h, n, 64)).astype(np.float32), "fp16") for _ in range(3))
    out = np.zeros((s, n, h * 64), np.uint16)
    ms = ctypes.c_float(0)
    _lib.check(lib.m3r_attention_fwd(0, 1, _lib.ptr(to16(q, "fp16")), _lib.ptr(to16(k, "fp16")),
                                     _lib.ptr(to16(v, "fp16")), _lib.ptr(out), s, h, n, n, 0.125, 1, ctypes.byref(ms)))
    sc = np.einsum("shqd,shkd->shqk", q.astype(np.float64), k.astype(np.float64)) * 0.125
    p = np.exp(sc - sc.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    ref = np.einsum("shqk,shkd->shqd", p, v.astype(np.float64)).transpose(0, 2, 1, 3).reshape(s, n, -1)
    return rel_l2(from16(out, "fp16"), ref) < 2e-3


def test_never_signalled_wait_times_out_and_gpu_stays_usable(lib):
    assert _attention_ok(lib)
    code = ctypes.c_int(-1)
    t0 = time.perf_counter()
    rc = lib.m3r_wait_selftest(0, 1_000_000, ctypes.byref(code))  # 1 ms limit
    dt = time.perf_counter() - t0
    assert rc == M3R_ERR_TIMEOUT, rc
    assert code.value == KDEV_TIMEOUT_MMA
    assert b"timed out" in lib.m3r_global_error()
    assert dt < 1.0, dt
    # the context is intact: a normal launch right after gives correct results
    assert _attention_ok(lib)
    rc = lib.m3r_wait_selftest(0, 3_000_000, ctypes.byref(code))  # and again, 3 ms
    assert rc == M3R_ERR_TIMEOUT and code.value == KDEV_TIMEOUT_MMA
    assert _attention_ok(lib)


def test_wait_selftest_rejects_bad_limits(lib):
    code = ctypes.c_int(0)
    assert lib.m3r_wait_selftest(0, 0, ctypes.byref(code)) == -1
    assert lib.m3r_wait_selftest(0, 20_000_000_000, ctypes.byref(code)) == -1


def test_engine_wait_limit_does_not_change_results(tmp_path):
    """A short (but sufficient) limit on a healthy pipeline: no wait runs out and the
    outputs are bit-identical to the default limit's."""
    from mast3r_runtime_b200 import NativeEngine, _lib, make_weights, save_safetensors, tiny_dims

    d = tiny_dims()
    path = save_safetensors(tmp_path / "u.safetensors", make_weights(d, seed=6, randomize_affine=True))
    rng = np.random.default_rng(3)
    img1 = rng.integers(0, 256, (2, 64, 96, 3), dtype=np.uint8)
    img2 = rng.integers(0, 256, (2, 64, 96, 3), dtype=np.uint8)
    eng = NativeEngine(d, (64, 96), [0], 2)
    eng.load(str(path))
    ref, _ = eng.infer_batch(img1, img2)
    _lib.check(eng.lib.m3r_set_wait_timeout(eng.h, 200_000_000), eng.h)  # 200 ms
    got, _ = eng.infer_batch(img1, img2)
    _lib.check(eng.lib.m3r_set_wait_timeout(eng.h, 0), eng.h)
    eng.close()
    for k in ref:
        np.testing.assert_array_equal(got[k], ref[k])
