"""Kernel parity on the GPU, through the C ABI (include/m3r_cuda.h).

GEMM / conv / attention are floating point: compared with float64 references computed
from the same bf16-rounded operands, tolerances stated per test.  The matcher is
compared with the oracle bit for bit (indices and confidences)."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import DTYPES, from16, matcher_inputs, rel_l2, round16, to16

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    from mast3r_runtime_b200 import _lib

    L = _lib.load()
    n = ctypes.c_int(0)
    _lib.check(L.m3r_device_count(ctypes.byref(n)))
    assert n.value > 0, "no CUDA device visible"
    return L


def P(a):
    return a.ctypes.data_as(ctypes.c_void_p)


# ---------------------------------------------------------------------------- GEMM
@pytest.mark.parametrize("pair", [0, 1], ids=["cta", "pair"])
@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("M,N,K,bn", [
    (128, 256, 64, 256),
    (300, 200, 136, 128),   # ragged M, N, K (TMA zero fill, epilogue masks)
    (389, 512, 1024, 256),
    (1000, 96, 96, 128),
    (2048, 768, 3072, 256),
])
def test_gemm_matches_fp64(lib, M, N, K, bn, dtype, pair):
    from mast3r_runtime_b200 import _lib

    rng = np.random.default_rng(M + N + K)
    a = round16(rng.standard_normal((M, K)).astype(np.float32), dtype)
    w = round16(rng.standard_normal((N, K)).astype(np.float32) * 0.05, dtype)
    bias = rng.standard_normal(N).astype(np.float32)
    c = np.zeros((M, N), np.float32)
    ms = ctypes.c_float(0)
    _lib.check(lib.m3r_gemm_test(0, DTYPES[dtype], P(to16(a, dtype)), P(to16(w, dtype)), P(bias), P(c), M, N, K, bn,
                                 pair, 2, ctypes.byref(ms)))
    ref = a.astype(np.float64) @ w.astype(np.float64).T + bias
    # fp32 accumulation of K exact 16-bit products: relative error ~ sqrt(K) * 2^-24
    assert rel_l2(c, ref) < 1e-5, rel_l2(c, ref)
    assert np.abs(c - ref).max() < 1e-4 * np.sqrt(K) * (np.abs(ref).max() + 1)


@pytest.mark.parametrize("pair", [0, 1], ids=["cta", "pair"])
@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("M,N,K,bn", [
    (128, 256, 64, 256),
    (300, 200, 136, 128),   # ragged M and N: zero-filled residual loads, clipped stores
    (389, 516, 256, 256),   # a last column unit 4 wide
    (1000, 96, 96, 128),    # second column group idle in every tile
    (2048, 768, 3072, 256),
    (4500, 1024, 1024, 256),  # several tiles per CTA: the residual ring crosses tiles
])
def test_gemm_residual_matches_fp64(lib, M, N, K, bn, dtype, pair):
    """c += A W^T + bias in place: the residual epilogue (TMA-loaded residual ring)."""
    from mast3r_runtime_b200 import _lib

    rng = np.random.default_rng(M * 7 + N + K)
    a = round16(rng.standard_normal((M, K)).astype(np.float32), dtype)
    w = round16(rng.standard_normal((N, K)).astype(np.float32) * 0.05, dtype)
    bias = rng.standard_normal(N).astype(np.float32)
    resid = (rng.standard_normal((M, N)) * 4).astype(np.float32)
    c = resid.copy()
    _lib.check(lib.m3r_gemm_resid_test(0, DTYPES[dtype], P(to16(a, dtype)), P(to16(w, dtype)), P(bias), P(c), M, N, K,
                                       bn, pair))
    ref = resid.astype(np.float64) + a.astype(np.float64) @ w.astype(np.float64).T + bias
    assert rel_l2(c, ref) < 1e-5, rel_l2(c, ref)
    assert np.abs(c - ref).max() < 1e-4 * np.sqrt(K) * (np.abs(ref).max() + 1)


def _upsample_ref(x, ho, wo):
    """Bilinear NHWC upsampling with half-pixel centres and clamped borders, float64 (the
    source coordinate (o + 0.5) * n_in / n_out - 0.5, clamped to [0, n_in - 1])."""
    n, hi, wi, c = x.shape

    def taps(n_in, n_out):
        s = np.maximum((np.arange(n_out) + 0.5) * (n_in / n_out) - 0.5, 0.0)
        i0 = np.minimum(np.floor(s).astype(np.int64), n_in - 1)
        i1 = np.minimum(i0 + 1, n_in - 1)
        return i0, i1, s - i0

    y0, y1, fy = taps(hi, ho)
    x0, x1, fx = taps(wi, wo)
    xd = x.astype(np.float64)
    fy = fy[None, :, None, None]
    fx = fx[None, None, :, None]
    top = xd[:, y0][:, :, x0] * (1 - fx) + xd[:, y0][:, :, x1] * fx
    bot = xd[:, y1][:, :, x0] * (1 - fx) + xd[:, y1][:, :, x1] * fx
    return top * (1 - fy) + bot * fy


def _within_one_ulp(got, ref, mag, dtype):
    """Every value within one unit in the last place of the 16-bit type (one rounding of an
    fp32 result) plus the fp32 accumulation error, bounded by 2^-21 x the sum of the terms'
    magnitudes `mag` (it matters only where the terms cancel)."""
    mant = 10 if dtype == "fp16" else 7
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(ref), 2.0 ** -14))) - mant)
    tol = ulp + 2.0 ** -21 * mag
    err = np.abs(got.astype(np.float64) - ref)
    assert np.all(err <= tol), float((err / tol).max())


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("n,h,w,c", [(2, 5, 7, 16), (1, 24, 32, 256), (3, 9, 4, 8)])
def test_resize2x_matches_fp64(lib, n, h, w, c, dtype):
    """The DPT head's 2x upsampling kernel (sliding rows, mixed-precision weights)."""
    from mast3r_runtime_b200 import _lib

    rng = np.random.default_rng(n * 100 + h + w + c)
    x = round16(rng.standard_normal((n, h, w, c)).astype(np.float32) * 3, dtype)
    y = np.zeros((n, 2 * h, 2 * w, c), np.uint16)
    _lib.check(lib.m3r_resize2x_test(0, DTYPES[dtype], P(to16(x, dtype)), n, h, w, c, P(y)))
    _within_one_ulp(from16(y, dtype), _upsample_ref(x, 2 * h, 2 * w), _upsample_ref(np.abs(x), 2 * h, 2 * w), dtype)


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("n,H,W,c,pyramid", [
    (2, 48, 64, 32, True),    # levels at 1/2, 1/4, 1/8: the mixed-precision kernel
    (1, 96, 128, 256, True),  # the ViT-L 512x384 head's sizes, one image
    (2, 40, 56, 16, False),   # other ratios: the general kernel
])
def test_dpt_fuse_matches_fp64(lib, n, H, W, c, pyramid, dtype):
    """f0 + up(f1) + up(f2) + up(f3) (the DPT fusion kernel)."""
    from mast3r_runtime_b200 import _lib

    rng = np.random.default_rng(n + H + W + c)
    sizes = [(H // 2, W // 2), (H // 4, W // 4), (H // 8, W // 8)] if pyramid else [(H // 2, W // 2), (7, 9), (3, 5)]
    f0 = round16(rng.standard_normal((n, H, W, c)).astype(np.float32), dtype)
    fs = [round16(rng.standard_normal((n, hh, ww, c)).astype(np.float32), dtype) for hh, ww in sizes]
    out = np.zeros((n, H, W, c), np.uint16)
    args = []
    for f, (hh, ww) in zip(fs, sizes):
        args += [P(to16(f, dtype)), hh, ww]
    _lib.check(lib.m3r_dpt_fuse_test(0, DTYPES[dtype], P(to16(f0, dtype)), *args, n, H, W, c, P(out)))
    ref = f0.astype(np.float64) + sum(_upsample_ref(f, H, W) for f in fs)
    got = from16(out, dtype)
    if pyramid:
        mag = np.abs(f0).astype(np.float64) + sum(_upsample_ref(np.abs(f), H, W) for f in fs)
        _within_one_ulp(got, ref, mag, dtype)
    else:
        # fp32 interpolation weights that are not exact in 16 bits: one 16-bit rounding plus
        # fp32 arithmetic, judged against the sum's magnitude
        tol = (2.0 ** -10 if dtype == "fp16" else 2.0 ** -7) * (np.abs(ref) + 1.0)
        assert np.all(np.abs(got - ref) <= tol)


def _conv3_ref(x, w, b):
    n, h, wd, c = x.shape
    co = w.shape[0]
    xp = np.pad(x.astype(np.float64), ((0, 0), (1, 1), (1, 1), (0, 0)))
    out = np.zeros((n, h, wd, co))
    for t in range(9):
        dy, dx = t // 3, t % 3
        out += xp[:, dy:dy + h, dx:dx + wd, :] @ w[:, t, :c].T.astype(np.float64)
    return out + b


@pytest.mark.parametrize("pair", [0, 1], ids=["cta", "pair"])
@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("n,h,wd,c,cout,bn", [
    (2, 8, 16, 64, 128, 128),
    (1, 12, 12, 96, 256, 256),    # channels padded to 128; w = 12 -> 4-wide boxes
    (2, 5, 32, 192, 128, 128),    # h not a multiple of the box height
    (1, 16, 128, 128, 128, 128),
    (2, 3, 256, 64, 128, 128),    # 128-pixel row tiles: wide-box taps on CTA pairs, borders
    (1, 5, 384, 192, 128, 128),
])
def test_conv3_matches_fp64(lib, n, h, wd, c, cout, bn, dtype, pair):
    from mast3r_runtime_b200 import _lib

    rng = np.random.default_rng(n * 1000 + h + wd + c)
    cpad = (c + 63) // 64 * 64
    x = round16(rng.standard_normal((n, h, wd, c)).astype(np.float32), dtype)
    w = np.zeros((cout, 9, cpad), np.float32)
    w[:, :, :c] = round16(rng.standard_normal((cout, 9, c)).astype(np.float32) * 0.05, dtype)
    b = rng.standard_normal(cout).astype(np.float32)
    y = np.zeros((n, h, wd, cout), np.float32)
    _lib.check(lib.m3r_conv3_test(0, DTYPES[dtype], P(to16(x, dtype)), P(to16(w, dtype)), P(b), P(y), n, h, wd, c,
                                  cout, bn, pair))
    ref = _conv3_ref(x, w, b)
    assert rel_l2(y, ref) < 1e-5, rel_l2(y, ref)


# ---------------------------------------------------------------------------- attention
def _attn_ref(q, k, v, scale):
    s = np.einsum("shqd,shkd->shqk", q.astype(np.float64), k.astype(np.float64)) * scale
    s -= s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    o = np.einsum("shqk,shkd->shqd", p, v.astype(np.float64))
    return o.transpose(0, 2, 1, 3).reshape(q.shape[0], q.shape[2], -1)  # [s, tok, h*64]


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("s,h,nq,nk", [
    (2, 3, 128, 128),
    (3, 2, 576, 576),   # 4.5 tiles: masked key tail, partial query tile
    (1, 1, 24, 24),     # tiny grid of the golden model
    (2, 2, 200, 300),   # nq != nk (cross attention)
    (2, 12, 768, 768),
])
def test_attention_matches_fp64(lib, s, h, nq, nk, dtype):
    from mast3r_runtime_b200 import _lib

    rng = np.random.default_rng(s * 100 + h + nq + nk)
    q = round16(rng.standard_normal((s, h, nq, 64)).astype(np.float32), dtype)
    k = round16(rng.standard_normal((s, h, nk, 64)).astype(np.float32), dtype)
    v = round16(rng.standard_normal((s, h, nk, 64)).astype(np.float32), dtype)
    out = np.zeros((s, nq, h * 64), np.uint16)
    ms = ctypes.c_float(0)
    _lib.check(lib.m3r_attention_fwd(0, DTYPES[dtype], P(to16(q, dtype)), P(to16(k, dtype)), P(to16(v, dtype)),
                                     P(out), s, h, nq, nk, 0.125, 2, ctypes.byref(ms)))
    got = from16(out, dtype)
    ref = _attn_ref(q, k, v, 0.125)
    # 16-bit probabilities and output: |err| ~ 2^-8 (bf16) / 2^-11 (fp16) of the output scale
    tol = 1e-2 if dtype == "bf16" else 2e-3
    err = rel_l2(got, ref)
    assert err < tol, err
    assert np.abs(got - ref).max() < 3 * tol * (np.abs(ref).max() + 1e-3)


# ---------------------------------------------------------------------------- matcher
def _nn_gpu(lib, a, b):
    from mast3r_runtime_b200 import _lib

    n1, d = a.shape
    n2 = b.shape[0]
    nn12 = np.zeros(n1, np.int32)
    nn21 = np.zeros(n2, np.int32)
    b12 = np.zeros(n1, np.float32)
    ms = ctypes.c_float(0)
    _lib.check(lib.m3r_match_nn(0, P(np.ascontiguousarray(a)), P(np.ascontiguousarray(b)), n1, n2, d, P(nn12),
                                P(nn21), P(b12), ctypes.byref(ms)))
    return nn12, nn21, b12


@pytest.mark.parametrize("n1,n2,d", [(4096, 4096, 24), (1000, 3001, 24), (777, 555, 64), (300, 260, 256), (5, 7, 24)])
def test_match_argmax_bit_exact(lib, oracle_lib, n1, n2, d):
    rng = np.random.default_rng(n1 + n2 + d)
    a = rng.standard_normal((n1, d)).astype(np.float32)
    b = rng.standard_normal((n2, d)).astype(np.float32)
    b[: n2 // 4] = a[rng.integers(0, n1, n2 // 4)]          # exact copies: ties between rows
    a[n1 // 2: n1 // 2 + 3] = a[0]                          # duplicated rows: column ties
    g12, g21, gb = _nn_gpu(lib, a, b)
    an = oracle_lib.normalize(a)
    bn = oracle_lib.normalize(b)
    o12, ob12, o21, _ = oracle_lib.argmax(an, bn)
    np.testing.assert_array_equal(g12, o12)
    np.testing.assert_array_equal(g21, o21)
    assert gb.tobytes() == ob12.tobytes()


@pytest.mark.parametrize("kind", ["a_row0", "b_row0", "a_row9", "inf"])
def test_match_argmax_non_finite(lib, oracle_lib, kind):
    """NaN / inf descriptors: row 0 (column 0) seeds every column (row) and a NaN seed
    is never replaced; NaN elsewhere never wins (matching.cpp:128-155)."""
    rng = np.random.default_rng(3)
    a = rng.standard_normal((700, 24)).astype(np.float32)
    b = rng.standard_normal((900, 24)).astype(np.float32)
    if kind == "a_row0":
        a[0, 5] = np.nan
    elif kind == "b_row0":
        b[0] = np.nan
        a[300] = np.nan
    elif kind == "a_row9":
        a[9] = np.nan
        b[400, 1] = np.nan
    else:
        a[4, 0] = np.inf
        b[7, 3] = -np.inf
    g12, g21, gb = _nn_gpu(lib, a, b)
    o12, ob12, o21, _ = oracle_lib.argmax(oracle_lib.normalize(a), oracle_lib.normalize(b))
    np.testing.assert_array_equal(g12, o12)
    np.testing.assert_array_equal(g21, o21)
    nan = np.isnan(ob12)
    np.testing.assert_array_equal(np.isnan(gb), nan)
    assert gb[~nan].tobytes() == ob12[~nan].tobytes()


@pytest.fixture(scope="module")
def matcher_engine(lib):
    from mast3r_runtime_b200 import NativeEngine, tiny_dims

    return NativeEngine(tiny_dims(), (32, 32), [0], 1)


@pytest.mark.parametrize("h,w,d,top_k,recip,thr", [
    (64, 64, 24, 512, True, 0.5),      # top-k selection path
    (48, 64, 24, 4096, True, 0.0),     # all candidates, i order
    (48, 64, 24, 100, False, 0.5),
    (16, 16, 64, 512, True, 0.0),
    (192, 256, 24, 512, True, 0.5),    # a quarter of the 512x384 map
])
def test_match_bit_exact_vs_oracle(matcher_engine, oracle_lib, h, w, d, top_k, recip, thr):
    a, b = matcher_inputs(h, w, d, h * w + d)
    r = matcher_engine.match(a, b, top_k=top_k, reciprocal=recip, confidence_threshold=thr)
    o = oracle_lib.match(a, b, top_k=top_k, reciprocal=recip, confidence_threshold=thr)
    np.testing.assert_array_equal(r.idx_1, o["idx_1"])
    np.testing.assert_array_equal(r.idx_2, o["idx_2"])
    assert r.confidence.tobytes() == o["confidence"].tobytes()
    np.testing.assert_array_equal(r.pts2d_1, o["pts2d_1"])
    np.testing.assert_array_equal(r.pts2d_2, o["pts2d_2"])


@pytest.mark.parametrize("h,w,d,top_k,recip,thr", [
    (48, 64, 24, 512, True, 1.5),      # top-k cut of the weighted similarities
    (40, 64, 24, 4096, True, 0.0),     # all candidates
    (32, 32, 24, 200, False, 1.0),
])
def test_match_confidence_weighted_bit_exact_vs_oracle(matcher_engine, oracle_lib, h, w, d, top_k, recip, thr):
    """conf_1[i] * conf_2[j] weighting (matching.cpp:110-119) and the pts3d gather
    (matching.py:144-152), bit for bit."""
    a, b = matcher_inputs(h, w, d, h + w + 1)
    rng = np.random.default_rng(h * w)
    c1 = (1.0 + 2.0 * rng.random((h, w))).astype(np.float32)
    c2 = (1.0 + 2.0 * rng.random((h, w))).astype(np.float32)
    q1 = rng.standard_normal((h, w, 3)).astype(np.float32)
    q2 = rng.standard_normal((h, w, 3)).astype(np.float32)
    kw = dict(top_k=top_k, reciprocal=recip, confidence_threshold=thr, conf_1=c1, conf_2=c2, pts3d_1=q1, pts3d_2=q2)
    r = matcher_engine.match(a, b, **kw)
    o = oracle_lib.match(a, b, **kw)
    assert len(o["idx_1"]) > 0
    np.testing.assert_array_equal(r.idx_1, o["idx_1"])
    np.testing.assert_array_equal(r.idx_2, o["idx_2"])
    assert r.confidence.tobytes() == o["confidence"].tobytes()
    np.testing.assert_array_equal(r.pts3d_1, o["pts3d_1"])
    np.testing.assert_array_equal(r.pts3d_2, o["pts3d_2"])
    # weighting changes the result (the test is not vacuous)
    u = matcher_engine.match(a, b, top_k=top_k, reciprocal=recip, confidence_threshold=thr)
    assert len(u.idx_1) != len(r.idx_1) or not np.array_equal(u.confidence, r.confidence)


def test_match_kats_gpu(matcher_engine):
    rng = np.random.default_rng(0)
    desc = rng.random((8, 8, 64)).astype(np.float32)
    r = matcher_engine.match(desc, desc, reciprocal=True, confidence_threshold=0.0)
    np.testing.assert_array_equal(r.idx_1, r.idx_2)
    assert len(r.idx_1) == 64
    same = np.ones((4, 4, 24), np.float32)
    r = matcher_engine.match(same, same, top_k=16, confidence_threshold=0.0)
    assert r.idx_1.tolist() == [0] and r.idx_2.tolist() == [0]
    d1 = np.zeros((4, 4, 64), np.float32)
    d1[..., :32] = 1.0
    d2 = np.zeros((4, 4, 64), np.float32)
    d2[..., 32:] = 1.0
    assert len(matcher_engine.match(d1, d2, confidence_threshold=0.5).idx_1) == 0
    empty = np.zeros((0, 0, 64), np.float32)
    assert len(matcher_engine.match(empty, empty).idx_1) == 0
    one = rng.random((1, 1, 64)).astype(np.float32)
    assert len(matcher_engine.match(one, one).idx_1) <= 1


# ---------------------------------------------------------------------------- preprocessing
@pytest.mark.parametrize("h,w,oh,ow", [(300, 200, 224, 224), (336, 336, 336, 336), (1024, 768, 512, 512),
                                       (97, 131, 64, 64), (640, 360, 336, 336), (480, 640, 384, 512),
                                       (768, 1024, 384, 512), (50, 70, 64, 96)])
def test_resize_crop_bit_exact_vs_oracle(lib, oracle_lib, h, w, oh, ow):
    """Resize + centre crop of csrc/cpu/preprocessing.cpp (the oracle's restatement is pinned
    to the reference's own C++ by tests/test_oracle.py), bit for bit, including upscaling
    and rectangular model sizes."""
    from mast3r_runtime_b200 import _lib

    img = np.random.default_rng(h + w).integers(0, 256, (h, w, 3), dtype=np.uint8)
    out = np.zeros((oh, ow, 3), np.uint8)
    _lib.check(lib.m3r_resize_crop_test(0, P(img), h, w, P(out), oh, ow))
    np.testing.assert_array_equal(out, oracle_lib.resize_crop(img, (oh, ow)))
