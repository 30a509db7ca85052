"""Generate the golden fixtures in this directory by running the REFERENCE code.

Run where the reference tree is available, naming it in M3R_REFERENCE:

    M3R_REFERENCE=<reference tree> python tests/golden/make_golden.py [--large]

It imports the reference's own numpy model classes
(mast3r_runtime/backends/python/{croco_encoder,croco_decoder,rope2d,mast3r_model}.py)
and matcher (mast3r_runtime/backends/matching.py), and loads the reference's C++
matcher (csrc/cpu/matching.cpp, compiled into oracle/_ref by oracle/Makefile).  The
outputs are written as small .npz fixtures; the inputs are regenerated from seeds
by the tests, so only outputs and seeds are stored.

Fixtures
  model_tiny.npz    encoder / decoder / reference-CPU-head outputs of a tiny CroCo
                    model (seeded weights, randomised biases and LayerNorm params)
                    on a seeded 64x96 image pair, plus RoPE2D of a seeded tensor
  matcher.npz       reference reciprocal_match (C++ and numpy) on seeded descriptor
                    maps, several (top_k, reciprocal, threshold) settings
  matcher_large.npz (--large) the reference's C++ reciprocal_match on a 180 x 256
                    map (N = 46,080, 24-d, the config-4 input recipe): the largest N
                    its int-typed N * N similarity allocation accepts is 46,340
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
REF = Path(os.environ["M3R_REFERENCE"]) if os.environ.get("M3R_REFERENCE") else None

MODEL_SEED = 1234
IMAGE_SEED = (42, 43)
IMAGE_HW = (64, 96)
LARGE_CASE = (180, 256, 24, 5, 512, True, 0.5)  # (H, W, D, seed, top_k, reciprocal, threshold)
MATCH_CASES = [  # (H, W, D, seed, top_k, reciprocal, threshold)
    (8, 8, 24, 7, 512, True, 0.5),
    (16, 24, 24, 8, 64, True, 0.0),
    (16, 24, 24, 9, 64, False, 0.5),
    (12, 16, 64, 10, 16, True, 0.0),
    (4, 4, 64, 11, 512, True, 0.9),
    (20, 20, 24, 12, 100, True, 0.3),
]


def tiny_dims():
    sys.path.insert(0, str(ROOT))
    from mast3r_runtime_b200.weights import tiny_dims as td

    return td()


def seeded_images():
    imgs = []
    for s in IMAGE_SEED:
        rng = np.random.default_rng(s)
        imgs.append(rng.integers(0, 256, (*IMAGE_HW, 3), dtype=np.uint8))
    return imgs


def matcher_inputs(h, w, d, seed):
    """Set B is 30% noisy (sigma 0.05) copies of set A rows, the rest fresh Gaussian."""
    rng = np.random.default_rng(seed)
    n = h * w
    a = rng.standard_normal((n, d)).astype(np.float32)
    b = rng.standard_normal((n, d)).astype(np.float32)
    m = int(0.3 * n)
    dst = rng.permutation(n)[:m]
    src = rng.permutation(n)[:m]
    b[dst] = a[src] + np.float32(0.05) * rng.standard_normal((m, d)).astype(np.float32)
    return a.reshape(h, w, d), b.reshape(h, w, d)


def main_large():
    """matcher_large.npz from the reference's own C++ matcher (oracle/_ref)."""
    sys.path.insert(0, str(ROOT))
    import oracle

    if oracle.ref_lib() is None:
        oracle.build()
    h, w, d, seed, top_k, recip, thr = LARGE_CASE
    a, b = matcher_inputs(h, w, d, seed)
    r = oracle.ref_match(a, b, top_k=top_k, reciprocal=recip, confidence_threshold=thr)
    if r is None:
        raise SystemExit("oracle/_ref is not built: the reference tree is needed")
    np.savez_compressed(HERE / "matcher_large.npz", case=np.array([h, w, d, seed, top_k, int(recip),
                                                                    int(round(thr * 1000))]), **r)
    print("wrote", HERE / "matcher_large.npz", len(r["idx_1"]), "matches")


def main():
    sys.dont_write_bytecode = True
    if REF is None:
        raise SystemExit("set M3R_REFERENCE to the reference tree")
    sys.path.insert(0, str(REF))
    sys.path.insert(0, str(ROOT))
    from mast3r_runtime.backends.python.croco_decoder import CroCoDecoder
    from mast3r_runtime.backends.python.croco_encoder import CroCoEncoder
    from mast3r_runtime.backends.python.mast3r_model import MASt3RDPTHead
    from mast3r_runtime.backends.python.python_engine import PythonEngine  # noqa: F401 (import check)
    from mast3r_runtime.backends.python.rope2d import PositionGetter, RoPE2D
    from mast3r_runtime.backends import matching as ref_matching

    from mast3r_runtime_b200.weights import make_weights
    import oracle

    d = tiny_dims()
    w = make_weights(d, seed=MODEL_SEED, randomize_affine=True)
    img1, img2 = seeded_images()

    # python_engine.py:176-188 preprocessing (no resize: inputs have the model size)
    def prep(img):
        x = img.astype(np.float32) / 255.0
        x = (x - np.array([0.485, 0.456, 0.406], np.float32)) / np.array([0.229, 0.224, 0.225], np.float32)
        return np.transpose(x, (2, 0, 1))[None]

    enc = CroCoEncoder(w, num_heads=d.enc_heads)
    dec = CroCoDecoder(w, num_heads=d.dec_heads)
    e1, p1 = enc(prep(img1))
    e2, p2 = enc(prep(img2))
    d1, d2 = dec(e1, e2, p1, p2)
    hg, wg = IMAGE_HW[0] // d.patch, IMAGE_HW[1] // d.patch
    h1 = MASt3RDPTHead(w, "downstream_head1")
    pts1, desc1, conf1 = h1(d1, e1, hg, wg, IMAGE_HW)

    rng = np.random.default_rng(5)
    t = rng.standard_normal((1, 2, hg * wg, 64)).astype(np.float32)
    pos = PositionGetter()(1, hg, wg)
    roped = RoPE2D(freq=100.0)(t, pos)

    np.savez_compressed(
        HERE / "model_tiny.npz",
        model_seed=MODEL_SEED, image_seeds=np.array(IMAGE_SEED), image_hw=np.array(IMAGE_HW),
        enc_1=e1[0].astype(np.float32), enc_2=e2[0].astype(np.float32),
        dec_1=d1[0].astype(np.float32), dec_2=d2[0].astype(np.float32),
        ref_simple_pts3d_1=pts1[0].astype(np.float32), ref_simple_conf_1=conf1[0].astype(np.float32),
        ref_simple_desc_1=desc1[0, :, :, :32].astype(np.float32),
        rope_in=t, rope_out=roped.astype(np.float32), positions=pos[0],
    )

    L = oracle.ref_lib()
    if L is None:
        oracle.build()
        L = oracle.ref_lib()
    store = {}
    for ci, (h, ww, dd, seed, top_k, recip, thr) in enumerate(MATCH_CASES):
        a, b = matcher_inputs(h, ww, dd, seed)
        r = oracle.ref_match(a, b, top_k=top_k, reciprocal=recip, confidence_threshold=thr)
        rn = ref_matching.reciprocal_match(a, b, top_k=top_k, reciprocal=recip, confidence_threshold=thr)
        for k, v in r.items():
            store[f"c{ci}_cpp_{k}"] = v
        store[f"c{ci}_np_idx_1"] = rn.idx_1
        store[f"c{ci}_np_idx_2"] = rn.idx_2
        store[f"c{ci}_np_confidence"] = rn.confidence
    store["cases"] = np.array([[h, ww, dd, s, k, int(r), int(round(t * 1000))] for h, ww, dd, s, k, r, t in MATCH_CASES])
    np.savez_compressed(HERE / "matcher.npz", **store)
    print("wrote", HERE / "model_tiny.npz", HERE / "matcher.npz")


if __name__ == "__main__":
    if REF is None:
        raise SystemExit("set M3R_REFERENCE to the reference tree")
    os.environ.setdefault("M3R_REFERENCE", str(REF))
    main_large() if "--large" in sys.argv[1:] else main()
