"""Multi-GPU paths (need >= 2 visible devices): pairs sharded over an engine's devices
give the same outputs as one device; the row-sharded matcher (column keys max-reduced
with NCCL) is bit-exact with the oracle, top-k cut included."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import matcher_inputs

pytestmark = pytest.mark.gpu


def _ndev():
    from mast3r_runtime_b200 import device_count

    return device_count()


@pytest.fixture(scope="module")
def two_gpus():
    n = _ndev()
    if n < 2:
        pytest.skip(f"{n} GPU visible: the multi-GPU paths need 2")
    return [0, 1]


@pytest.mark.parametrize("h,w,d,top_k,recip,thr", [
    (96, 128, 24, 512, True, 0.5),     # more candidates than top_k: per-shard top-k + merge
    (64, 64, 24, 4096, True, 0.0),     # all candidates, row order across shards
    (48, 64, 64, 200, False, 0.3),
])
def test_sharded_match_bit_exact(two_gpus, oracle_lib, h, w, d, top_k, recip, thr):
    from mast3r_runtime_b200 import NativeEngine, tiny_dims

    eng = NativeEngine(tiny_dims(), (32, 32), two_gpus, 1)
    a, b = matcher_inputs(h, w, d, 77 + h)
    r = eng.match(a, b, top_k=top_k, reciprocal=recip, confidence_threshold=thr)
    o = oracle_lib.match(a, b, top_k=top_k, reciprocal=recip, confidence_threshold=thr)
    np.testing.assert_array_equal(r.idx_1, o["idx_1"])
    np.testing.assert_array_equal(r.idx_2, o["idx_2"])
    assert r.confidence.tobytes() == o["confidence"].tobytes()
    eng.close()


def test_sharded_confidence_weighted_match_bit_exact(two_gpus, oracle_lib):
    from mast3r_runtime_b200 import NativeEngine, tiny_dims

    eng = NativeEngine(tiny_dims(), (32, 32), two_gpus, 1)
    a, b = matcher_inputs(96, 128, 24, 91)
    rng = np.random.default_rng(4)
    c1 = (1.0 + rng.random((96, 128))).astype(np.float32)
    c2 = (1.0 + rng.random((96, 128))).astype(np.float32)
    kw = dict(top_k=512, reciprocal=True, confidence_threshold=1.0, conf_1=c1, conf_2=c2)
    r = eng.match(a, b, **kw)
    o = oracle_lib.match(a, b, **kw)
    np.testing.assert_array_equal(r.idx_1, o["idx_1"])
    np.testing.assert_array_equal(r.idx_2, o["idx_2"])
    assert r.confidence.tobytes() == o["confidence"].tobytes()
    eng.close()


def test_pairs_sharded_over_devices_match_single_device(two_gpus, tmp_path):
    from mast3r_runtime_b200 import NativeEngine, make_weights, save_safetensors, tiny_dims

    d = tiny_dims()
    path = save_safetensors(tmp_path / "u.safetensors", make_weights(d, seed=4, randomize_affine=True))
    rng = np.random.default_rng(1)
    img1 = rng.integers(0, 256, (5, 64, 96, 3), dtype=np.uint8)
    img2 = rng.integers(0, 256, (5, 64, 96, 3), dtype=np.uint8)
    one = NativeEngine(d, (64, 96), [0], 5)
    one.load(str(path))
    ref, _ = one.infer_batch(img1, img2)
    two = NativeEngine(d, (64, 96), two_gpus, 3)
    two.load(str(path))
    got, _ = two.infer_batch(img1, img2)
    for k in ref:
        np.testing.assert_array_equal(got[k], ref[k])
    one.close()
    two.close()
