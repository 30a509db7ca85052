"""ORACLE -- test infrastructure only.

CPU restatements of the reference (Aedelon/mast3r-runtime) two-view inference
path and reciprocal matcher, plus loaders for the reference's own CPU kernels
compiled from its sources (``oracle/_ref``).  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import this
package, and only as the checker: the product path (``mast3r_runtime_b200``)
never imports it.

Contents
  matcher.c   / liboracle.so       blocked C restatement of csrc/cpu/matching.cpp
  _ref/libm3r_ref.so               reference csrc/cpu/{matching,attention}.cpp
  model.py                         numpy restatement of the CroCo encoder/decoder
                                   (backends/python/croco_*.py) and the 24-d
                                   MASt3R head (csrc/mps/mpsgraph_engine.mm)
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_LIB = None
_REF = None

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")


def build() -> None:
    """Compile liboracle.so (and oracle/_ref when the reference tree exists)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        path = HERE / "liboracle.so"
        if not path.exists():
            build()
        L = ctypes.CDLL(str(path))
        L.oracle_normalize.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int]
        L.oracle_normalize.restype = None
        L.oracle_argmax.argtypes = [_f32p, _f32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                                    ctypes.c_int64, ctypes.c_int64, _i32p, _f32p, _i32p, _f32p]
        L.oracle_argmax.restype = None
        L.oracle_match.argtypes = [_f32p, _f32p, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                   _i64p, _i64p, _f32p, _f32p, _f32p, ctypes.c_void_p, ctypes.c_void_p]
        L.oracle_match.restype = ctypes.c_int64
        _opt = ctypes.c_void_p  # optional float arrays (None = absent)
        L.oracle_match_w.argtypes = [_f32p, _f32p, _opt, _opt, _opt, _opt, ctypes.c_int64, ctypes.c_int,
                                     ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                     _i64p, _i64p, _f32p, _f32p, _f32p, _opt, _opt, ctypes.c_void_p,
                                     ctypes.c_void_p]
        L.oracle_match_w.restype = ctypes.c_int64
        L.oracle_argmax_w.argtypes = [_f32p, _f32p, _opt, _opt, ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                                      ctypes.c_int64, ctypes.c_int64, _i32p, _f32p, _i32p, _f32p]
        L.oracle_argmax_w.restype = None
        L.oracle_attention.argtypes = [_f32p, _f32p, _f32p, _f32p, ctypes.c_int64, ctypes.c_int,
                                       ctypes.c_int, ctypes.c_int, ctypes.c_float]
        L.oracle_attention.restype = None
        _u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
        L.oracle_resize_crop.argtypes = [_u8p, ctypes.c_int, ctypes.c_int, _u8p, ctypes.c_int, ctypes.c_int]
        L.oracle_resize_crop.restype = None
        L.oracle_normalize_chw.argtypes = [_u8p, ctypes.c_int, ctypes.c_int, _f32p]
        L.oracle_normalize_chw.restype = None
        _LIB = L
    return _LIB


def ref_lib() -> ctypes.CDLL | None:
    """The reference's own csrc/cpu kernels, or None when oracle/_ref is absent."""
    global _REF
    if _REF is None:
        path = HERE / "_ref" / "libm3r_ref.so"
        if not path.exists():
            return None
        L = ctypes.CDLL(str(path))
        L.ref_reciprocal_match.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                           ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                           _i64p, _i64p, _f32p, _f32p, _f32p]
        L.ref_reciprocal_match.restype = ctypes.c_int64
        L.ref_reciprocal_match_conf.argtypes = [_f32p, _f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int,
                                                ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                                _i64p, _i64p, _f32p, _f32p, _f32p]
        L.ref_reciprocal_match_conf.restype = ctypes.c_int64
        L.ref_preprocess.argtypes = [np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS"), ctypes.c_int,
                                     ctypes.c_int, ctypes.c_int, _f32p]
        L.ref_preprocess.restype = None
        L.ref_normalize.argtypes = [_f32p, ctypes.c_int, ctypes.c_int]
        L.ref_normalize.restype = None
        L.ref_multi_head_attention.argtypes = [_f32p, _f32p, _f32p, _f32p, ctypes.c_int,
                                               ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.ref_multi_head_attention.restype = None
        _REF = L
    return _REF


def normalize(desc: np.ndarray) -> np.ndarray:
    """csrc/cpu/matching.cpp:22-44 on a copy of ``desc`` ([..., D] float32)."""
    d = desc.shape[-1]
    out = np.ascontiguousarray(desc, dtype=np.float32).reshape(-1, d).copy()
    lib().oracle_normalize(out, out.shape[0], d)
    return out.reshape(desc.shape)


def argmax(a_norm: np.ndarray, b_norm: np.ndarray, row0: int = 0, row1: int | None = None, conf_1=None,
           conf_2=None):
    """Row/column arg-max of a_norm . b_norm^T (already normalised), lowest index on ties.

    Returns (nn12, best12, nn21, best21); nn12/best12 are only filled in [row0, row1).
    """
    a = np.ascontiguousarray(a_norm, dtype=np.float32)
    b = np.ascontiguousarray(b_norm, dtype=np.float32)
    n1, d = a.shape
    n2 = b.shape[0]
    row1 = n1 if row1 is None else row1
    nn12 = np.zeros(n1, np.int32)
    b12 = np.zeros(n1, np.float32)
    nn21 = np.zeros(n2, np.int32)
    b21 = np.zeros(n2, np.float32)
    c1 = None if conf_1 is None else np.ascontiguousarray(conf_1, np.float32).reshape(n1)
    c2 = None if conf_2 is None else np.ascontiguousarray(conf_2, np.float32).reshape(n2)
    lib().oracle_argmax_w(a, b, None if c1 is None else c1.ctypes.data_as(ctypes.c_void_p),
                          None if c2 is None else c2.ctypes.data_as(ctypes.c_void_p), n1, n2, d, row0, row1,
                          nn12, b12, nn21, b21)
    return nn12, b12, nn21, b21


def _opt32(x, n):
    if x is None:
        return None, None
    a = np.ascontiguousarray(x, dtype=np.float32).reshape(n, -1)
    return a, a.ctypes.data_as(ctypes.c_void_p)


def match(desc_1: np.ndarray, desc_2: np.ndarray, top_k: int = 512, reciprocal: bool = True,
          confidence_threshold: float = 0.5, with_nn: bool = False, conf_1=None, conf_2=None,
          pts3d_1=None, pts3d_2=None):
    """Restated reciprocal_match on [H, W, D] maps (csrc/cpu/matching.cpp:85-237), with the
    confidence weighting of :110-119 when conf_1 and conf_2 ([H, W]) are given and the
    pts3d gather of matching.py:144-152 when pts3d_1 and pts3d_2 ([H, W, 3]) are.

    Returns a dict with idx_1, idx_2 (int64), confidence, pts2d_1, pts2d_2, pts3d_1,
    pts3d_2 (float32) and, when ``with_nn``, nn_12 / nn_21 (int32).
    """
    h, w, d = desc_1.shape
    n = h * w
    a = np.ascontiguousarray(desc_1, dtype=np.float32).reshape(n, d)
    b = np.ascontiguousarray(desc_2, dtype=np.float32).reshape(n, d)
    cap = max(min(top_k, n), 1)
    idx1 = np.zeros(cap, np.int64)
    idx2 = np.zeros(cap, np.int64)
    conf = np.zeros(cap, np.float32)
    p1 = np.zeros(cap * 2, np.float32)
    p2 = np.zeros(cap * 2, np.float32)
    nn12 = np.zeros(max(n, 1), np.int32)
    nn21 = np.zeros(max(n, 1), np.int32)
    weighted = conf_1 is not None and conf_2 is not None
    c1, c1p = _opt32(conf_1 if weighted else None, n)
    c2, c2p = _opt32(conf_2 if weighted else None, n)
    q1, q1p = _opt32(pts3d_1 if pts3d_2 is not None else None, n)
    q2, q2p = _opt32(pts3d_2 if pts3d_1 is not None else None, n)
    o1 = np.zeros(cap * 3, np.float32)
    o2 = np.zeros(cap * 3, np.float32)
    m = lib().oracle_match_w(a, b, c1p, c2p, q1p, q2p, n, d, w, top_k, int(bool(reciprocal)),
                             float(confidence_threshold), idx1, idx2, conf, p1, p2,
                             o1.ctypes.data_as(ctypes.c_void_p), o2.ctypes.data_as(ctypes.c_void_p),
                             nn12.ctypes.data if with_nn else None,
                             nn21.ctypes.data if with_nn else None)
    if m < 0:
        raise ValueError("oracle_match: bad arguments")
    out = {
        "idx_1": idx1[:m].copy(), "idx_2": idx2[:m].copy(), "confidence": conf[:m].copy(),
        "pts2d_1": p1[: 2 * m].reshape(m, 2).copy(), "pts2d_2": p2[: 2 * m].reshape(m, 2).copy(),
        "pts3d_1": o1[: 3 * m].reshape(m, 3).copy(), "pts3d_2": o2[: 3 * m].reshape(m, 3).copy(),
    }
    if with_nn:
        out["nn_12"] = nn12[:n].copy()
        out["nn_21"] = nn21[:n].copy()
    return out


def ref_match(desc_1: np.ndarray, desc_2: np.ndarray, top_k: int = 512, reciprocal: bool = True,
              confidence_threshold: float = 0.5, conf_1=None, conf_2=None):
    """The reference's own reciprocal_match (oracle/_ref), or None when unavailable.

    It materialises the N x N similarity matrix: keep N small.
    """
    L = ref_lib()
    if L is None:
        return None
    h, w, d = desc_1.shape
    n = h * w
    a = np.ascontiguousarray(desc_1, dtype=np.float32).reshape(n, d)
    b = np.ascontiguousarray(desc_2, dtype=np.float32).reshape(n, d)
    cap = max(min(top_k, n), 1)
    idx1 = np.zeros(cap, np.int64)
    idx2 = np.zeros(cap, np.int64)
    conf = np.zeros(cap, np.float32)
    p1 = np.zeros(cap * 2, np.float32)
    p2 = np.zeros(cap * 2, np.float32)
    if conf_1 is not None and conf_2 is not None:
        c1 = np.ascontiguousarray(conf_1, np.float32).reshape(n)
        c2 = np.ascontiguousarray(conf_2, np.float32).reshape(n)
        m = L.ref_reciprocal_match_conf(a, b, c1, c2, h, w, d, top_k, int(bool(reciprocal)),
                                        float(confidence_threshold), idx1, idx2, conf, p1, p2)
    else:
        m = L.ref_reciprocal_match(a, b, h, w, d, top_k, int(bool(reciprocal)),
                                   float(confidence_threshold), idx1, idx2, conf, p1, p2)
    return {
        "idx_1": idx1[:m].copy(), "idx_2": idx2[:m].copy(), "confidence": conf[:m].copy(),
        "pts2d_1": p1[: 2 * m].reshape(m, 2).copy(), "pts2d_2": p2[: 2 * m].reshape(m, 2).copy(),
    }


def resize_crop(img: np.ndarray, out_hw) -> np.ndarray:
    """Restated resize + centre crop of csrc/cpu/preprocessing.cpp:29-63, 84-129 (uint8
    [h, w, 3] -> uint8 [H, W, 3]; the reference's target is square, H == W)."""
    src = np.ascontiguousarray(img, np.uint8)
    out = np.zeros((int(out_hw[0]), int(out_hw[1]), 3), np.uint8)
    lib().oracle_resize_crop(src, src.shape[0], src.shape[1], out, out.shape[0], out.shape[1])
    return out


def normalize_chw(img: np.ndarray) -> np.ndarray:
    """preprocessing.cpp:65-82: (v / 255 - mean) / std, [h, w, 3] uint8 -> [3, h, w] float32."""
    src = np.ascontiguousarray(img, np.uint8)
    out = np.zeros((3, src.shape[0], src.shape[1]), np.float32)
    lib().oracle_normalize_chw(src, src.shape[0], src.shape[1], out)
    return out


def ref_preprocess(img: np.ndarray, res: int):
    """The reference's own Preprocessor(res).process (oracle/_ref), or None when unavailable."""
    L = ref_lib()
    if L is None:
        return None
    src = np.ascontiguousarray(img, np.uint8)
    out = np.zeros((3, res, res), np.float32)
    L.ref_preprocess(src, src.shape[0], src.shape[1], res, out)
    return out


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float) -> np.ndarray:
    """fp32 softmax(Q K^T * scale) V over [..., N, dh] slices (C, OpenMP)."""
    dh = q.shape[-1]
    nq, nk = q.shape[-2], k.shape[-2]
    qs = np.ascontiguousarray(q, np.float32).reshape(-1, nq, dh)
    ks = np.ascontiguousarray(k, np.float32).reshape(-1, nk, dh)
    vs = np.ascontiguousarray(v, np.float32).reshape(-1, nk, dh)
    o = np.zeros_like(qs)
    lib().oracle_attention(qs, ks, vs, o, qs.shape[0], nq, nk, dh, float(scale))
    return o.reshape(q.shape)


def cpu_count() -> int:
    return len(os.sched_getaffinity(0))
