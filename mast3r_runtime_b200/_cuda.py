"""Drop-in ``_cuda`` backend module for mast3r-runtime, over the C ABI of libm3r_cuda.so.

The reference dispatcher selects BackendType.CUDA by importing
``mast3r_runtime.backends._cuda`` (mast3r_runtime/backends/__init__.py:173-179) and
expects, as its CPU binding provides (csrc/cpu/bindings.cpp:207-253):

  module functions   is_available(), get_device_name(), get_compute_capability()
                     (mast3r_runtime/backends/__init__.py:46-51, 129-138)
  CUDAEngine(variant, resolution, precision, num_threads)            (:204-215)
      load(path), is_ready(), name(), warmup(n)                       (native_wrapper.py:40-64)
      infer(img1, img2) -> .pts3d_1/2 [H,W,3] .desc_1/2 [H,W,24] .conf_1/2 [H,W] .timing
                                                                      (native_wrapper.py:84-97)
      match(desc_1, desc_2, top_k=, reciprocal=, confidence_threshold=)
          -> .idx_1/2 int64 [K] .pts2d_1/2 [K,2] .pts3d_1/2 [K,3] .confidence [K] .timing
                                                                      (native_wrapper.py:122-140)

``install()`` registers this module under that name (the reference's own tests use the
same sys.modules technique, tests/integration/test_backends.py:30-49), so the
unmodified reference package picks it up.

Errors follow the reference bindings: bad shapes raise ValueError / RuntimeError
(pybind11 maps std::runtime_error to RuntimeError, csrc/cpu/bindings.cpp:18-20).
There is no CPU fallback: without the built library or a GPU every compute call raises.

Precision: the reference's Precision.FP16 (its default) and FP32 (core/config.py:42-48)
run fp16 tensor-core operands, "bf16" runs bf16 operands; both accumulate in fp32 and
keep the residual stream and every output in fp32.
"""

from __future__ import annotations

import ctypes
import os
import sys
import time
from types import SimpleNamespace

import numpy as np

from . import _lib
from .weights import VARIANTS, ModelDims


# ----------------------------------------------------------------------------- module functions
def is_available() -> bool:
    """True when libm3r_cuda.so loads and at least one CUDA device is visible (never raises)."""
    try:
        lib = _lib.load()
        n = ctypes.c_int(0)
        return lib.m3r_device_count(ctypes.byref(n)) == 0 and n.value > 0
    except Exception:
        return False


def device_count() -> int:
    lib = _lib.load()
    n = ctypes.c_int(0)
    _lib.check(lib.m3r_device_count(ctypes.byref(n)))
    return n.value


def get_device_name(device: int = 0) -> str:
    lib = _lib.load()
    buf = ctypes.create_string_buffer(256)
    _lib.check(lib.m3r_device_info(device, buf, 256, None, None))
    return buf.value.decode()


def get_compute_capability(device: int = 0) -> tuple[int, int]:
    lib = _lib.load()
    ma, mi = ctypes.c_int(0), ctypes.c_int(0)
    _lib.check(lib.m3r_device_info(device, None, 0, ctypes.byref(ma), ctypes.byref(mi)))
    return (ma.value, mi.value)


def make_config(dims: ModelDims, image_hw: tuple[int, int], devices=(0,), max_pairs: int = 1,
                dtype: int = _lib.DTYPE_F16, head: int = _lib.HEAD_MAST3R24) -> _lib.M3RConfig:
    c = _lib.M3RConfig()
    c.patch = dims.patch
    c.enc_dim, c.enc_depth, c.enc_heads, c.enc_mlp = dims.enc_dim, dims.enc_depth, dims.enc_heads, dims.enc_mlp
    c.dec_dim, c.dec_depth, c.dec_heads, c.dec_mlp = dims.dec_dim, dims.dec_depth, dims.dec_heads, dims.dec_mlp
    c.lf_hidden = dims.lf_hidden
    c.desc_dim = _lib.HEAD_DESC_DIM[int(head)]
    c.head = int(head)
    c.img_h, c.img_w = int(image_hw[0]), int(image_hw[1])
    devices = list(devices)
    if len(devices) > _lib.M3R_MAX_DEVICES:
        raise ValueError("too many devices")
    c.n_devices = len(devices)
    for i, d in enumerate(devices):
        c.devices[i] = int(d)
    c.max_pairs = int(max_pairs)
    c.dtype = int(dtype)
    return c


def _env_devices() -> list[int]:
    s = os.environ.get("M3R_CUDA_DEVICES", "").strip()
    if not s:
        return [0]
    return [int(x) for x in s.split(",") if x.strip()]


class NativeEngine:
    """One libm3r_cuda engine: fixed model dims, image size, device list and launch size."""

    def __init__(self, dims: ModelDims, image_hw, devices=(0,), max_pairs: int = 1, dtype: int = _lib.DTYPE_F16,
                 head: int = _lib.HEAD_MAST3R24):
        self.lib = _lib.load()
        self.dims = dims
        self.image_hw = (int(image_hw[0]), int(image_hw[1]))
        self.devices = list(devices)
        self.max_pairs = int(max_pairs)
        self.dtype = int(dtype)
        self.dtype_name = _lib.DTYPE_NAMES[self.dtype]
        self.head = int(head)
        self.desc_dim = _lib.HEAD_DESC_DIM[self.head]  # output descriptor channels
        cfg = make_config(dims, self.image_hw, self.devices, self.max_pairs, self.dtype, self.head)
        # pinned output sets recycled across infer_batch calls that allocate their outputs
        self._pool = _lib.OutputPool(lambda n: self._out_arrays(n, alloc=_lib.pinned_empty))
        h = ctypes.c_void_p()
        _lib.check(self.lib.m3r_create(ctypes.byref(cfg), ctypes.byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            self.lib.m3r_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def load(self, path: str) -> None:
        _lib.check(self.lib.m3r_load(self.h, str(path).encode()), self.h)

    def is_ready(self) -> bool:
        return bool(self.lib.m3r_is_ready(self.h))

    def _out_arrays(self, n: int, alloc=np.empty):
        H, W = self.image_hw
        D = self.desc_dim
        return {
            "pts3d_1": alloc((n, H, W, 3), np.float32), "pts3d_2": alloc((n, H, W, 3), np.float32),
            "desc_1": alloc((n, H, W, D), np.float32), "desc_2": alloc((n, H, W, D), np.float32),
            "conf_1": alloc((n, H, W), np.float32), "conf_2": alloc((n, H, W), np.float32),
        }

    def _check_images(self, img1, img2):
        img1 = np.ascontiguousarray(img1, dtype=np.uint8)
        img2 = np.ascontiguousarray(img2, dtype=np.uint8)
        if img1.ndim == 3:
            img1, img2 = img1[None], img2[None]
        if img1.ndim != 4 or img1.shape[-1] != 3 or img1.shape != img2.shape:
            raise ValueError(f"Expected [H, W, 3] (or [N, H, W, 3]) uint8 image pairs, got {img1.shape} / {img2.shape}")
        if tuple(img1.shape[1:3]) != self.image_hw:
            raise ValueError(f"image size {img1.shape[1:3]} differs from the engine's {self.image_hw}")
        return img1, img2

    def infer_batch(self, img1, img2, out=None):
        """[N, H, W, 3] uint8 pairs -> dict of [N, ...] fp32 outputs and a timing dict.

        Without `out` the outputs are views of recycled page-locked buffers (OutputPool):
        the device copies land in them directly."""
        img1, img2 = self._check_images(img1, img2)
        n = img1.shape[0]
        o = out if out is not None else self._pool.get(n)
        t = np.zeros(len(_lib.TIMING_KEYS), np.float32)
        rc = self.lib.m3r_infer(self.h, _lib.ptr(img1), _lib.ptr(img2), n,
                                _lib.ptr(o["pts3d_1"]), _lib.ptr(o["pts3d_2"]), _lib.ptr(o["desc_1"]),
                                _lib.ptr(o["desc_2"]), _lib.ptr(o["conf_1"]), _lib.ptr(o["conf_2"]), _lib.ptr(t))
        _lib.check(rc, self.h)
        return o, dict(zip(_lib.TIMING_KEYS, map(float, t)))

    def infer_any(self, img1, img2):
        """One pair of uint8 [h, w, 3] images of any size: resized and centre-cropped to the
        engine's size on the device (the reference's preprocessing, csrc/cpu/preprocessing.cpp
        and python_engine.py:158-174), then the forward pass.  Returns ({k: [1, ...]}, timing)."""
        a = np.ascontiguousarray(img1, dtype=np.uint8)
        b = np.ascontiguousarray(img2, dtype=np.uint8)
        if a.ndim != 3 or a.shape[2] != 3 or b.ndim != 3 or b.shape[2] != 3:
            raise ValueError(f"Expected [H, W, 3] uint8 images, got {a.shape} / {b.shape}")
        o = self._pool.get(1)
        t = np.zeros(len(_lib.TIMING_KEYS), np.float32)
        rc = self.lib.m3r_infer_any(self.h, _lib.ptr(a), a.shape[0], a.shape[1], _lib.ptr(b), b.shape[0], b.shape[1],
                                    _lib.ptr(o["pts3d_1"]), _lib.ptr(o["pts3d_2"]), _lib.ptr(o["desc_1"]),
                                    _lib.ptr(o["desc_2"]), _lib.ptr(o["conf_1"]), _lib.ptr(o["conf_2"]), _lib.ptr(t))
        _lib.check(rc, self.h)
        return o, dict(zip(_lib.TIMING_KEYS, map(float, t)))

    def load_retrieval(self, path: str) -> None:
        """Whitening weights (prewhiten.m, prewhiten.p) of the retrieval head
        (csrc/mps/mpsgraph_engine.mm:758-787); the encoder weights are the loaded model's."""
        _lib.check(self.lib.m3r_load_retrieval(self.h, str(path).encode()), self.h)

    def encode_retrieval(self, images):
        """[n, H, W, 3] (or [H, W, 3]) uint8 images of the model size -> (features
        [n, N, enc_dim], attention [n, N]) fp32: the encoder output whitened as (x - m) P and
        the per-token L2 weights (mpsgraph_engine.mm:1030-1117)."""
        imgs = np.ascontiguousarray(images, dtype=np.uint8)
        if imgs.ndim == 3:
            imgs = imgs[None]
        if imgs.ndim != 4 or tuple(imgs.shape[1:]) != (*self.image_hw, 3):
            raise ValueError(f"Expected [N, {self.image_hw[0]}, {self.image_hw[1]}, 3] uint8 images, got {imgs.shape}")
        n = imgs.shape[0]
        ntok = (self.image_hw[0] // self.dims.patch) * (self.image_hw[1] // self.dims.patch)
        feats = np.empty((n, ntok, self.dims.enc_dim), np.float32)
        attn = np.empty((n, ntok), np.float32)
        t = np.zeros(len(_lib.TIMING_KEYS), np.float32)
        _lib.check(self.lib.m3r_encode_retrieval(self.h, _lib.ptr(imgs), n, _lib.ptr(feats), _lib.ptr(attn),
                                                 _lib.ptr(t)), self.h)
        return feats, attn

    # device-resident stages (throughput measurement)
    def stage(self, img1, img2):
        img1, img2 = self._check_images(img1, img2)
        _lib.check(self.lib.m3r_stage_inputs(self.h, _lib.ptr(img1), _lib.ptr(img2), img1.shape[0]), self.h)
        return img1.shape[0]

    def run_resident(self, n: int) -> float:
        ms = ctypes.c_float(0)
        _lib.check(self.lib.m3r_run_resident(self.h, n, ctypes.byref(ms)), self.h)
        return ms.value

    def fetch(self, n: int, out=None):
        o = out if out is not None else self._out_arrays(n)
        _lib.check(self.lib.m3r_fetch_outputs(self.h, n, _lib.ptr(o["pts3d_1"]), _lib.ptr(o["pts3d_2"]),
                                              _lib.ptr(o["desc_1"]), _lib.ptr(o["desc_2"]),
                                              _lib.ptr(o["conf_1"]), _lib.ptr(o["conf_2"])), self.h)
        return o

    def set_profiling(self, on: bool):
        _lib.check(self.lib.m3r_set_profiling(self.h, int(bool(on))), self.h)

    def profile(self) -> dict:
        a = np.zeros(8, np.float64)
        _lib.check(self.lib.m3r_get_profile(self.h, _lib.ptr(a)), self.h)
        keys = ("gemm_ms", "gemm_flop", "attn_ms", "attn_flop", "other_ms", "gemm_launches", "attn_launches",
                "other_launches")
        return dict(zip(keys, map(float, a)))

    def profile_ops(self) -> dict:
        """{op: {"ms", "flop", "launches"}} of the last profiled pass, in launch order."""
        need = ctypes.c_int(0)
        _lib.check(self.lib.m3r_get_profile_ops(self.h, None, 0, ctypes.byref(need)), self.h)
        buf = ctypes.create_string_buffer(max(need.value, 1))
        _lib.check(self.lib.m3r_get_profile_ops(self.h, buf, len(buf), None), self.h)
        ops = {}
        for line in buf.value.decode().splitlines():
            name, ms, flop, launches = line.split("\t")
            ops[name] = {"ms": float(ms), "flop": float(flop), "launches": int(launches)}
        return ops

    def match(self, desc_1, desc_2, top_k=512, reciprocal=True, confidence_threshold=0.5, conf_1=None, conf_2=None,
              pts3d_1=None, pts3d_2=None):
        """reciprocal_match (backends/matching.py:53-165): conf_1 / conf_2 [H, W] weight every
        similarity by conf_1[i] * conf_2[j] (both needed); pts3d_1 / pts3d_2 [H, W, 3] give the
        3-D points of the matches (zeros without them)."""
        d1 = np.ascontiguousarray(desc_1, dtype=np.float32)
        d2 = np.ascontiguousarray(desc_2, dtype=np.float32)
        if d1.ndim != 3 or d2.ndim != 3:
            raise RuntimeError("Expected [H, W, D] arrays")
        if d1.shape != d2.shape:
            raise ValueError(f"descriptor maps differ in shape: {d1.shape} vs {d2.shape}")
        H, W, D = d1.shape
        weighted = conf_1 is not None and conf_2 is not None
        c1 = np.ascontiguousarray(conf_1, dtype=np.float32).reshape(H * W) if weighted else None
        c2 = np.ascontiguousarray(conf_2, dtype=np.float32).reshape(H * W) if weighted else None
        have3 = pts3d_1 is not None and pts3d_2 is not None
        q1 = np.ascontiguousarray(pts3d_1, dtype=np.float32).reshape(H * W, 3) if have3 else None
        q2 = np.ascontiguousarray(pts3d_2, dtype=np.float32).reshape(H * W, 3) if have3 else None
        n = H * W
        top_k = int(top_k)
        if top_k < 0:
            raise ValueError("top_k must be >= 0")
        cap = max(min(top_k, n), 1)
        idx1 = np.zeros(cap, np.int64)
        idx2 = np.zeros(cap, np.int64)
        conf = np.zeros(cap, np.float32)
        p1 = np.zeros((cap, 2), np.float32)
        p2 = np.zeros((cap, 2), np.float32)
        o1 = np.zeros((cap, 3), np.float32)
        o2 = np.zeros((cap, 3), np.float32)
        m = ctypes.c_int(0)
        t = np.zeros(len(_lib.TIMING_KEYS), np.float32)
        if n == 0 or D == 0:
            m.value = 0
        else:
            rc = self.lib.m3r_match_ex(self.h, _lib.ptr(d1), _lib.ptr(d2), _lib.ptr(c1), _lib.ptr(c2), _lib.ptr(q1),
                                       _lib.ptr(q2), H, W, D, top_k, int(bool(reciprocal)), float(confidence_threshold),
                                       _lib.ptr(idx1), _lib.ptr(idx2), _lib.ptr(conf), _lib.ptr(p1), _lib.ptr(p2),
                                       _lib.ptr(o1), _lib.ptr(o2), ctypes.byref(m), _lib.ptr(t))
            _lib.check(rc, self.h)
        k = m.value
        return SimpleNamespace(
            idx_1=idx1[:k].copy(), idx_2=idx2[:k].copy(), pts2d_1=p1[:k].copy(), pts2d_2=p2[:k].copy(),
            pts3d_1=o1[:k].copy(), pts3d_2=o2[:k].copy(),
            confidence=conf[:k].copy(),
            timing={"match_ms": float(t[7]), "kernel_ms": float(t[6]), "normalize_ms": float(t[0]),
                    "argmax_ms": float(t[1]), "select_ms": float(t[2])},
        )


# ----------------------------------------------------------------------------- the drop-in engine
class CUDAEngine:
    """``mast3r_runtime.backends._cuda.CUDAEngine``: the object NativeEngineWrapper drives.

    Model dimensions come from ``variant`` (core/config.py:19-28 names); the model input
    is ``resolution`` x ``resolution`` (the reference engines' convention) or
    ``image_size`` (any multiple of the patch, e.g. (384, 512)).  Images of another size
    are resized and centre-cropped to it on the device, as the reference preprocesses
    them.  Devices: M3R_CUDA_DEVICES (default "0").
    ``head``: "mast3r24" (the MASt3R DPT + local-feature head, 24-d L2-normalised
    descriptors) or "ref_simple" (the reference's CPU head MASt3RDPTHead,
    backends/python/mast3r_model.py:86-156: 256-d raw descriptors, convs at patch-grid
    resolution, bilinear upsampling).
    """

    def __init__(self, variant: str = "dune_vit_small_336", resolution: int = 336, precision: str = "fp16",
                 num_threads: int = 4, image_size: tuple[int, int] | None = None, devices=None,
                 head: str = "mast3r24"):
        if variant not in VARIANTS:
            raise RuntimeError(f"Unknown model variant: {variant}")
        self.variant = variant
        self.dims = VARIANTS[variant]
        self.precision = str(getattr(precision, "value", precision))
        self.dtype = _lib.dtype_for_precision(self.precision)
        self.num_threads = int(num_threads)
        self.image_hw = tuple(image_size) if image_size is not None else (int(resolution), int(resolution))
        self.devices = list(devices) if devices is not None else _env_devices()
        if head not in _lib.HEADS:
            raise RuntimeError(f"Unknown head: {head} (mast3r24 or ref_simple)")
        self.head = _lib.HEADS[head]
        self._engines: dict[tuple, NativeEngine] = {}
        self._path: str | None = None
        self._matcher: NativeEngine | None = None
        p = self.dims.patch
        if self.image_hw[0] % p or self.image_hw[1] % p:
            raise RuntimeError(f"resolution {self.image_hw} must be a multiple of the patch size {p}")

    # --- NativeEngineWrapper contract
    def name(self) -> str:
        try:
            dev = get_device_name(self.devices[0])
        except Exception:
            dev = "unavailable"
        return f"CUDA sm_100a ({self.variant}, {dev})"

    def load(self, path: str) -> None:
        path = str(path)
        if not os.path.exists(path):
            raise RuntimeError(f"weights file not found: {path}")
        self._engines.clear()
        self._path = path
        self._engine(self.image_hw, 1)

    def is_ready(self) -> bool:
        return self._path is not None and any(e.is_ready() for e in self._engines.values())

    def warmup(self, num_iterations: int = 3) -> None:
        rng = np.random.default_rng(42)
        H, W = self.image_hw
        dummy = rng.integers(0, 255, (H, W, 3), dtype=np.uint8)
        for _ in range(int(num_iterations)):
            self.infer(dummy, dummy)

    def infer(self, img1, img2):
        """native.infer (native_wrapper.py:84-97).  Images of another size than the engine's
        are resized and centre-cropped to it on the device, as the reference's engines
        preprocess them (csrc/cpu/preprocessing.cpp:29-63)."""
        img1 = np.asarray(img1)
        img2 = np.asarray(img2)
        if img1.ndim != 3 or img1.shape[2] != 3 or img2.ndim != 3 or img2.shape[2] != 3:
            raise RuntimeError("Expected [H, W, 3] uint8 array")
        if tuple(img1.shape[:2]) == self.image_hw and tuple(img2.shape[:2]) == self.image_hw:
            out, timing = self.infer_batch(img1[None], img2[None])
        else:
            out, timing = self._engine(self.image_hw, 1).infer_any(img1, img2)
        return SimpleNamespace(**{k: v[0] for k, v in out.items()}, timing=timing)

    def infer_batch(self, img1, img2):
        """[N, H, W, 3] pairs -> dict of [N, ...] outputs, timing (pairs sharded over devices).
        Pairs of another size than the engine's are preprocessed on the device one by one
        (infer_any), as infer does."""
        img1 = np.asarray(img1)
        img2 = np.asarray(img2)
        n = img1.shape[0]
        if tuple(img1.shape[1:3]) != self.image_hw or tuple(img2.shape[1:3]) != self.image_hw:
            eng = self._engine(self.image_hw, 1)
            parts = [eng.infer_any(img1[i], img2[i]) for i in range(n)]
            out = {k: np.concatenate([p[0][k] for p in parts]) for k in parts[0][0]}
            timing = {k: sum(p[1][k] for p in parts) for k in parts[0][1]}
            return out, timing
        per_dev = max(1, min(int(os.environ.get("M3R_PAIRS_PER_GPU", "64")), -(-n // len(self.devices))))
        eng = self._engine(self.image_hw, per_dev)
        return eng.infer_batch(img1, img2)

    def match(self, desc_1, desc_2, top_k: int = 512, reciprocal: bool = True, confidence_threshold: float = 0.5,
              conf_1=None, conf_2=None, pts3d_1=None, pts3d_2=None):
        """The wrapper's match (native_wrapper.py:99-140); also takes the reference matcher's
        optional conf_* / pts3d_* maps (backends/matching.py:53-63), which the wrapper itself
        does not pass on."""
        if self._matcher is None:
            # matching needs no weights: a minimal engine provides the device context
            self._matcher = next(iter(self._engines.values()), None) or NativeEngine(
                self.dims, (self.dims.patch * 2, self.dims.patch * 2), self.devices[:1], 1, self.dtype)
        t0 = time.perf_counter()
        r = self._matcher.match(desc_1, desc_2, top_k=top_k, reciprocal=reciprocal,
                                confidence_threshold=confidence_threshold, conf_1=conf_1, conf_2=conf_2,
                                pts3d_1=pts3d_1, pts3d_2=pts3d_2)
        r.timing["match_ms"] = (time.perf_counter() - t0) * 1000.0
        return r

    # --- retrieval (MPSGraphEngine::load_retrieval / encode_retrieval, mpsgraph_engine.mm:758-1117)
    def load_retrieval(self, path: str) -> None:
        self._retrieval_path = str(path)
        self._engine(self.image_hw, 1).load_retrieval(self._retrieval_path)

    def encode_retrieval(self, img):
        """One image -> SimpleNamespace(features [N, enc_dim], attention [N], num_patches,
        feature_dim) (the fields of the reference's RetrievalResult); other sizes are
        resized and centre-cropped first, as for infer."""
        img = np.asarray(img)
        if tuple(img.shape[:2]) != self.image_hw:
            raise RuntimeError(f"encode_retrieval takes {self.image_hw} images (resize them first)")
        eng = self._engine(self.image_hw, 1)
        if getattr(self, "_retrieval_path", None) is None:
            raise RuntimeError("retrieval weights are not loaded (call load_retrieval(path) first)")
        feats, attn = eng.encode_retrieval(img)
        return SimpleNamespace(features=feats[0], attention=attn[0], num_patches=feats.shape[1],
                               feature_dim=feats.shape[2])

    # --- internals
    def _engine(self, hw, max_pairs: int) -> NativeEngine:
        if self._path is None:
            raise RuntimeError("engine is not loaded (call load(path) first)")
        key = (tuple(hw), max_pairs)
        eng = self._engines.get(key)
        if eng is None:
            # drop engines of the same size but another launch size, to bound memory
            for k in [k for k in self._engines if k[0] == tuple(hw)]:
                self._engines.pop(k).close()
            eng = NativeEngine(self.dims, hw, self.devices, max_pairs, self.dtype, self.head)
            eng.load(self._path)
            if getattr(self, "_retrieval_path", None):
                eng.load_retrieval(self._retrieval_path)
            self._engines[key] = eng
        return eng


def install() -> None:
    """Register this module as ``mast3r_runtime.backends._cuda`` (BackendType.CUDA)."""
    sys.modules["mast3r_runtime.backends._cuda"] = sys.modules[__name__]
