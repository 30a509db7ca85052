"""The oracle is pinned before it is trusted: its restatements are checked against the
golden fixtures that tests/golden/make_golden.py produced by running the reference's own
code, and against the reference's known-answer tests (tests/unit/test_matching.py)."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import GOLDEN, matcher_inputs, rel_l2


# ---------------------------------------------------------------------------- model restatement
@pytest.fixture(scope="module")
def tiny_model():
    from make_golden import seeded_images
    from mast3r_runtime_b200.weights import make_weights, tiny_dims
    from oracle import model as om

    g = np.load(GOLDEN / "model_tiny.npz")
    d = tiny_dims()
    w = make_weights(d, seed=int(g["model_seed"]), randomize_affine=True)
    m = om.Model(w, d)
    img1, img2 = seeded_images()
    return g, m, img1, img2


def test_encoder_matches_reference(tiny_model):
    from oracle import model as om

    g, m, img1, img2 = tiny_model
    e1, _ = m.encode(om.preprocess(img1))
    e2, _ = m.encode(om.preprocess(img2))
    assert rel_l2(e1, g["enc_1"]) < 1e-5
    assert rel_l2(e2, g["enc_2"]) < 1e-5


def test_decoder_matches_reference(tiny_model):
    from oracle import model as om

    g, m, img1, img2 = tiny_model
    e1, grid = m.encode(om.preprocess(img1))
    e2, _ = m.encode(om.preprocess(img2))
    (d1, _), (d2, _) = m.decode(e1, e2, grid)
    assert rel_l2(d1, g["dec_1"]) < 1e-5
    assert rel_l2(d2, g["dec_2"]) < 1e-5


def test_ref_simple_head_matches_reference(tiny_model):
    from oracle import model as om

    g, m, img1, img2 = tiny_model
    e1, grid = m.encode(om.preprocess(img1))
    e2, _ = m.encode(om.preprocess(img2))
    (d1, _), _ = m.decode(e1, e2, grid)
    pts, desc, conf = m.ref_simple_head("downstream_head1", e1, d1, grid, tuple(g["image_hw"]))
    assert rel_l2(pts, g["ref_simple_pts3d_1"]) < 1e-5
    assert rel_l2(conf, g["ref_simple_conf_1"]) < 1e-5
    assert rel_l2(desc[..., :32], g["ref_simple_desc_1"]) < 1e-5


def test_rope_matches_reference():
    from oracle import model as om

    g = np.load(GOLDEN / "model_tiny.npz")
    cos, sin = om.rope_tables(g["positions"], 64)
    out = om.rope(g["rope_in"][0].astype(np.float64), cos, sin)
    assert rel_l2(out, g["rope_out"][0]) < 1e-6


def test_full_forward_outputs_are_sane(tiny_model):
    g, m, img1, img2 = tiny_model
    out = m.forward(img1, img2)
    H, W = g["image_hw"]
    for v in (1, 2):
        assert out[f"pts3d_{v}"].shape == (H, W, 3)
        assert out[f"conf_{v}"].shape == (H, W)
        assert out[f"desc_{v}"].shape == (H, W, 24)
        np.testing.assert_allclose(np.linalg.norm(out[f"desc_{v}"], axis=-1), 1.0, rtol=1e-6)
        assert np.isfinite(out[f"pts3d_{v}"]).all()


def test_bilinear_half_pixel_matches_closed_form():
    from oracle import model as om

    x = np.arange(4, dtype=np.float64).reshape(1, 4, 1)
    y = om.resize_bilinear(x, 1, 8)[0, :, 0]
    # PyTorch / MPSGraph align_corners=False: src = (i + 0.5) / 2 - 0.5, clamped at 0
    np.testing.assert_allclose(y, [0, 0.25, 0.75, 1.25, 1.75, 2.25, 2.75, 3.0])


# ---------------------------------------------------------------------------- matcher restatement
def test_matcher_golden_cpp_and_numpy(oracle_lib):
    z = np.load(GOLDEN / "matcher.npz")
    for ci, (h, w, d, seed, top_k, recip, thr_m) in enumerate(z["cases"]):
        a, b = matcher_inputs(int(h), int(w), int(d), int(seed))
        o = oracle_lib.match(a, b, top_k=int(top_k), reciprocal=bool(recip), confidence_threshold=thr_m / 1000.0)
        ref1, ref2, refc = z[f"c{ci}_cpp_idx_1"], z[f"c{ci}_cpp_idx_2"], z[f"c{ci}_cpp_confidence"]
        assert len(o["idx_1"]) == len(ref1)
        # same matches with bit-identical confidences (ordering of equal confidences is unspecified
        # in the reference's partial_sort, so compare as sets keyed by the pair)
        got = {(int(i), int(j)): c for i, j, c in zip(o["idx_1"], o["idx_2"], o["confidence"])}
        want = {(int(i), int(j)): c for i, j, c in zip(ref1, ref2, refc)}
        assert got.keys() == want.keys()
        assert all(np.float32(got[k]).tobytes() == np.float32(want[k]).tobytes() for k in got)
        # numpy reference: same match set (its confidences differ in the last bits: BLAS dot order)
        np_set = set(zip(z[f"c{ci}_np_idx_1"].tolist(), z[f"c{ci}_np_idx_2"].tolist()))
        assert len(np_set ^ set(got.keys())) <= max(2, len(got) // 50)
        # pts2d = (idx % W, idx // W)
        np.testing.assert_array_equal(o["pts2d_1"][:, 0], o["idx_1"] % w)
        np.testing.assert_array_equal(o["pts2d_1"][:, 1], o["idx_1"] // w)


def test_matcher_large_golden(oracle_lib):
    """The oracle at N = 46,080 against the reference C++ matcher's committed output."""
    z = np.load(GOLDEN / "matcher_large.npz")
    h, w, d, seed, top_k, recip, thr_m = (int(x) for x in z["case"])
    a, b = matcher_inputs(h, w, d, seed)
    o = oracle_lib.match(a, b, top_k=top_k, reciprocal=bool(recip), confidence_threshold=thr_m / 1000.0)
    got = {(int(i), int(j)): c for i, j, c in zip(o["idx_1"], o["idx_2"], o["confidence"])}
    want = {(int(i), int(j)): c for i, j, c in zip(z["idx_1"], z["idx_2"], z["confidence"])}
    assert len(got) == top_k and got.keys() == want.keys()
    assert all(np.float32(got[k]).tobytes() == np.float32(want[k]).tobytes() for k in got)


def test_matcher_against_reference_cpp_live(oracle_lib):
    if oracle_lib.ref_lib() is None:
        pytest.skip("oracle/_ref not built (reference tree absent)")
    for seed, (h, w, d) in enumerate([(24, 32, 24), (8, 8, 64), (3, 5, 24)]):
        a, b = matcher_inputs(h, w, d, 100 + seed)
        for recip in (True, False):
            o = oracle_lib.match(a, b, top_k=64, reciprocal=recip, confidence_threshold=0.0)
            r = oracle_lib.ref_match(a, b, top_k=64, reciprocal=recip, confidence_threshold=0.0)
            assert set(zip(o["idx_1"], o["idx_2"])) == set(zip(r["idx_1"], r["idx_2"]))


def _nan_cases():
    """Descriptor sets with NaN / inf entries: a NaN in row 0 of either set seeds every
    row (column) with a NaN that nothing replaces (matching.cpp:128-155); NaN elsewhere
    never wins a comparison."""
    cases = []
    for kind in ("a_row7", "b_row0", "a_row0", "inf"):
        a, b = matcher_inputs(6, 8, 24, 7)
        a, b = a.reshape(48, 24).copy(), b.reshape(48, 24).copy()
        if kind == "a_row7":
            a[7] = np.nan
        elif kind == "b_row0":
            b[0, 3] = np.nan
        elif kind == "a_row0":
            a[0, 0] = np.nan
            b[5] = np.nan
        else:
            a[3, 2] = np.inf
            b[9, 0] = -np.inf
        cases.append((kind, a.reshape(6, 8, 24), b.reshape(6, 8, 24)))
    return cases


@pytest.mark.parametrize("kind,a,b", _nan_cases(), ids=[c[0] for c in _nan_cases()])
def test_matcher_non_finite_matches_reference_cpp(oracle_lib, kind, a, b):
    if oracle_lib.ref_lib() is None:
        pytest.skip("oracle/_ref not built (reference tree absent)")
    for recip in (True, False):
        o = oracle_lib.match(a, b, top_k=64, reciprocal=recip, confidence_threshold=0.0)
        r = oracle_lib.ref_match(a, b, top_k=64, reciprocal=recip, confidence_threshold=0.0)
        got = {(int(i), int(j)): c for i, j, c in zip(o["idx_1"], o["idx_2"], o["confidence"])}
        want = {(int(i), int(j)): c for i, j, c in zip(r["idx_1"], r["idx_2"], r["confidence"])}
        assert got.keys() == want.keys(), kind
        assert all(np.float32(got[k]).tobytes() == np.float32(want[k]).tobytes() for k in got)


def _conf_case(seed, h=12, w=16, d=24):
    a, b = matcher_inputs(h, w, d, seed)
    rng = np.random.default_rng(seed + 1)
    c1 = (1.0 + rng.random((h, w))).astype(np.float32)      # confidences >= 1, as the head's 1 + exp
    c2 = (1.0 + rng.random((h, w))).astype(np.float32)
    p1 = rng.standard_normal((h, w, 3)).astype(np.float32)
    p2 = rng.standard_normal((h, w, 3)).astype(np.float32)
    return a, b, c1, c2, p1, p2


@pytest.mark.parametrize("recip", [True, False])
def test_matcher_confidence_weighted_matches_reference_cpp(oracle_lib, recip):
    """conf_1 / conf_2 weighting (matching.cpp:110-119) against the reference's own C++."""
    if oracle_lib.ref_lib() is None:
        pytest.skip("oracle/_ref not built (reference tree absent)")
    for seed in (3, 4):
        a, b, c1, c2, _, _ = _conf_case(seed)
        for thr in (0.0, 1.5):
            o = oracle_lib.match(a, b, top_k=64, reciprocal=recip, confidence_threshold=thr, conf_1=c1, conf_2=c2)
            r = oracle_lib.ref_match(a, b, top_k=64, reciprocal=recip, confidence_threshold=thr, conf_1=c1, conf_2=c2)
            got = {(int(i), int(j)): c for i, j, c in zip(o["idx_1"], o["idx_2"], o["confidence"])}
            want = {(int(i), int(j)): c for i, j, c in zip(r["idx_1"], r["idx_2"], r["confidence"])}
            assert got.keys() == want.keys() and len(got) > 0
            assert all(np.float32(got[k]).tobytes() == np.float32(want[k]).tobytes() for k in got)


def test_matcher_pts3d_gather_as_numpy_path(oracle_lib):
    """pts3d of the matches: pts3d_1[idx_1], pts3d_2[idx_2] (matching.py:144-152)."""
    a, b, c1, c2, p1, p2 = _conf_case(5)
    o = oracle_lib.match(a, b, top_k=64, confidence_threshold=0.0, conf_1=c1, conf_2=c2, pts3d_1=p1, pts3d_2=p2)
    np.testing.assert_array_equal(o["pts3d_1"], p1.reshape(-1, 3)[o["idx_1"]])
    np.testing.assert_array_equal(o["pts3d_2"], p2.reshape(-1, 3)[o["idx_2"]])
    z = oracle_lib.match(a, b, top_k=64, confidence_threshold=0.0)
    assert not z["pts3d_1"].any()


def _resized_dims(h, w, res):
    sc = max(np.float32(res) / np.float32(h), np.float32(res) / np.float32(w))
    return int(np.float32(h) * sc), int(np.float32(w) * sc)


@pytest.mark.parametrize("h,w,res", [(480, 640, 336), (300, 200, 224), (336, 336, 336), (1024, 768, 512),
                                     (97, 131, 64), (640, 360, 336)])
def test_preprocess_matches_reference_cpp(oracle_lib, h, w, res):
    """Resize + centre crop + normalise (csrc/cpu/preprocessing.cpp) bit for bit."""
    if oracle_lib.ref_lib() is None:
        pytest.skip("oracle/_ref not built (reference tree absent)")
    nh, nw = _resized_dims(h, w, res)
    if nh < res or nw < res:
        pytest.skip("the reference reads past its resized buffer here (truncated size below the target)")
    img = np.random.default_rng(h * w).integers(0, 256, (h, w, 3), dtype=np.uint8)
    got = oracle_lib.normalize_chw(oracle_lib.resize_crop(img, (res, res)))
    want = oracle_lib.ref_preprocess(img, res)
    assert got.tobytes() == want.tobytes()


def test_preprocess_identity_at_model_size(oracle_lib):
    img = np.random.default_rng(1).integers(0, 256, (64, 96, 3), dtype=np.uint8)
    np.testing.assert_array_equal(oracle_lib.resize_crop(img, (64, 96)), img)


def test_matcher_kats(oracle_lib):
    # tests/unit/test_matching.py:27-35: [3, 4] -> [0.6, 0.8]
    n = oracle_lib.normalize(np.array([[3.0, 4.0], [1.0, 0.0]], np.float32))
    np.testing.assert_allclose(n, [[0.6, 0.8], [1.0, 0.0]], rtol=1e-7)
    # zero vectors stay finite (matching.cpp:38 skips the division)
    assert np.isfinite(oracle_lib.normalize(np.zeros((1, 3), np.float32))).all()
    # identical descriptors -> identity matches (test_matching.py:234-240)
    rng = np.random.default_rng(0)
    desc = rng.random((8, 8, 64)).astype(np.float32)
    r = oracle_lib.match(desc, desc, reciprocal=True, confidence_threshold=0.0)
    np.testing.assert_array_equal(r["idx_1"], r["idx_2"])
    # top_k cap (test_matching.py:190-195)
    a, b = matcher_inputs(24, 24, 24, 3)
    assert len(oracle_lib.match(a, b, top_k=10)["idx_1"]) <= 10
    # reciprocal <= non-reciprocal; threshold monotone (test_matching.py:197-212)
    assert len(oracle_lib.match(a, b, reciprocal=True, top_k=4096)["idx_1"]) <= len(
        oracle_lib.match(a, b, reciprocal=False, top_k=4096)["idx_1"])
    assert len(oracle_lib.match(a, b, confidence_threshold=0.9)["idx_1"]) <= len(
        oracle_lib.match(a, b, confidence_threshold=0.0)["idx_1"])
    # orthogonal sets: nothing passes 0.5 (test_matching.py:341-355)
    d1 = np.zeros((4, 4, 64), np.float32)
    d1[..., :32] = 1.0
    d2 = np.zeros((4, 4, 64), np.float32)
    d2[..., 32:] = 1.0
    assert len(oracle_lib.match(d1, d2, confidence_threshold=0.5)["idx_1"]) == 0


def test_matcher_ties_lowest_index(oracle_lib):
    # all-equal descriptors: every similarity ties; nn_12 = 0 for every row, nn_21 = 0 for every column
    d = np.ones((4, 4, 24), np.float32)
    r = oracle_lib.match(d, d, top_k=16, confidence_threshold=0.0, with_nn=True)
    assert (r["nn_12"] == 0).all() and (r["nn_21"] == 0).all()
    assert r["idx_1"].tolist() == [0] and r["idx_2"].tolist() == [0]


def test_matcher_empty(oracle_lib):
    d = np.zeros((0, 0, 64), np.float32)
    assert len(oracle_lib.match(d, d)["idx_1"]) == 0
