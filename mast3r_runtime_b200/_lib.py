"""ctypes binding of libm3r_cuda.so (declarations in include/m3r_cuda.h).

Loading never silently falls back to anything: when the library is missing the
functions that need it raise RuntimeError.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libm3r_cuda.so"

M3R_OK = 0
ERRORS = {
    -1: "bad argument",
    -2: "I/O error",
    -3: "CUDA error",
    -4: "NCCL error",
    -5: "device wait timed out",
    -6: "invalid engine state",
    -7: "out of memory",
}
M3R_MAX_DEVICES = 16
TIMING_KEYS = ("preprocess_ms", "encoder_ms", "decoder_ms", "heads_ms", "h2d_ms", "d2h_ms", "inference_ms", "total_ms")


class M3RConfig(ctypes.Structure):
    _fields_ = [
        ("patch", ctypes.c_int), ("enc_dim", ctypes.c_int), ("enc_depth", ctypes.c_int),
        ("enc_heads", ctypes.c_int), ("enc_mlp", ctypes.c_int),
        ("dec_dim", ctypes.c_int), ("dec_depth", ctypes.c_int), ("dec_heads", ctypes.c_int),
        ("dec_mlp", ctypes.c_int), ("lf_hidden", ctypes.c_int), ("desc_dim", ctypes.c_int),
        ("img_h", ctypes.c_int), ("img_w", ctypes.c_int),
        ("n_devices", ctypes.c_int), ("devices", ctypes.c_int * M3R_MAX_DEVICES),
        ("max_pairs", ctypes.c_int), ("dtype", ctypes.c_int), ("head", ctypes.c_int),
    ]


HEAD_MAST3R24 = 0     # 24-d MASt3R DPT + local-feature head
HEAD_REF_SIMPLE = 1   # the reference's CPU head (256-d raw descriptors)
HEADS = {"mast3r24": HEAD_MAST3R24, "ref_simple": HEAD_REF_SIMPLE}
HEAD_DESC_DIM = {HEAD_MAST3R24: 24, HEAD_REF_SIMPLE: 256}

DTYPE_BF16 = 0
DTYPE_F16 = 1
DTYPE_NAMES = {DTYPE_BF16: "bf16", DTYPE_F16: "fp16"}


def dtype_for_precision(precision: str) -> int:
    """Map the reference's precision names (core/config.py:42-48) to the operand type:
    "fp16" (its default) and "fp32" run fp16 tensor cores, "bf16" runs bf16."""
    p = str(getattr(precision, "value", precision)).lower()
    if p == "bf16":
        return DTYPE_BF16
    if p in ("fp16", "fp32", "f16", "f32", "float16", "float32"):
        return DTYPE_F16
    raise ValueError(f"unsupported precision {precision!r} (fp32, fp16 or bf16)")


# exported symbol -> (restype, argtypes)
_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_I64 = ctypes.c_int64
SIGNATURES = {
    "m3r_version": (_I, []),
    "m3r_global_error": (ctypes.c_char_p, []),
    "m3r_device_count": (_I, [ctypes.POINTER(_I)]),
    "m3r_device_info": (_I, [_I, ctypes.c_char_p, _I, ctypes.POINTER(_I), ctypes.POINTER(_I)]),
    "m3r_create": (_I, [ctypes.POINTER(M3RConfig), ctypes.POINTER(_P)]),
    "m3r_destroy": (None, [_P]),
    "m3r_last_error": (ctypes.c_char_p, [_P]),
    "m3r_load": (_I, [_P, ctypes.c_char_p]),
    "m3r_is_ready": (_I, [_P]),
    "m3r_infer": (_I, [_P, _P, _P, _I, _P, _P, _P, _P, _P, _P, _P]),
    "m3r_match": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _F, _P, _P, _P, _P, _P, ctypes.POINTER(_I), _P]),
    "m3r_load_retrieval": (_I, [_P, ctypes.c_char_p]),
    "m3r_encode_retrieval": (_I, [_P, _P, _I, _P, _P, _P]),
    "m3r_infer_any": (_I, [_P, _P, _I, _I, _P, _I, _I, _P, _P, _P, _P, _P, _P, _P]),
    "m3r_resize2x_test": (_I, [_I, _I, _P, _I, _I, _I, _I, _P]),
    "m3r_dpt_fuse_test": (_I, [_I, _I, _P, _P, _I, _I, _P, _I, _I, _P, _I, _I, _I, _I, _I, _I, _P]),
    "m3r_resize_crop_test": (_I, [_I, _P, _I, _I, _P, _I, _I]),
    "m3r_match_ex": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _P, _P, _P, _P, _P, _P, _P,
                          ctypes.POINTER(_I), _P]),
    "m3r_stage_inputs": (_I, [_P, _P, _P, _I]),
    "m3r_run_resident": (_I, [_P, _I, ctypes.POINTER(_F)]),
    "m3r_fetch_outputs": (_I, [_P, _I, _P, _P, _P, _P, _P, _P]),
    "m3r_set_profiling": (_I, [_P, _I]),
    "m3r_get_profile": (_I, [_P, _P]),
    "m3r_get_profile_ops": (_I, [_P, ctypes.c_char_p, _I, ctypes.POINTER(_I)]),
    "m3r_host_alloc": (_P, [ctypes.c_size_t]),
    "m3r_host_free": (None, [_P]),
    "m3r_attention_fwd": (_I, [_I, _I, _P, _P, _P, _P, _I, _I, _I, _I, _F, _I, ctypes.POINTER(_F)]),
    "m3r_gemm_test": (_I, [_I, _I, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, ctypes.POINTER(_F)]),
    "m3r_gemm_resid_test": (_I, [_I, _I, _P, _P, _P, _P, _I, _I, _I, _I, _I]),
    "m3r_conv3_test": (_I, [_I, _I, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I]),
    "m3r_match_nn": (_I, [_I, _P, _P, _I64, _I64, _I, _P, _P, _P, ctypes.POINTER(_F)]),
    "m3r_match_nn_static": (_I, [_I, _P, _P, _I64, _I64, _I, _P, _P, _P, _P]),
    "m3r_set_wait_timeout": (_I, [_P, ctypes.c_ulonglong]),
    "m3r_wait_selftest": (_I, [_I, ctypes.c_ulonglong, ctypes.POINTER(_I)]),
    "m3r_check_checkpoint": (_I, [ctypes.POINTER(M3RConfig), ctypes.c_char_p]),
}

_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load libm3r_cuda.so (raises RuntimeError when it has not been built)."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(f"{LIB_PATH.name} is not built: run `python -m mast3r_runtime_b200.build`")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(rc: int, engine=None) -> None:
    """Map a status code to RuntimeError (ValueError for bad arguments)."""
    if rc == M3R_OK:
        return
    lib = load()
    msg = (lib.m3r_last_error(engine) if engine else lib.m3r_global_error()) or b""
    text = f"{ERRORS.get(rc, 'error')} ({rc}): {msg.decode(errors='replace')}"
    if rc == -1:
        raise ValueError(text)
    raise RuntimeError(text)


def ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def pinned_empty(shape, dtype) -> np.ndarray:
    """A numpy array in page-locked host memory (freed when the array is collected)."""
    lib = load()
    dtype = np.dtype(dtype)
    nbytes = int(np.prod(shape)) * dtype.itemsize
    p = lib.m3r_host_alloc(max(nbytes, 1))
    if not p:
        raise MemoryError("m3r_host_alloc failed")
    buf = (ctypes.c_uint8 * max(nbytes, 1)).from_address(p)
    arr = np.frombuffer(buf, dtype=np.uint8, count=nbytes).view(dtype).reshape(shape)

    class _Owner:
        def __init__(self, addr):
            self.addr = addr

        def __del__(self):
            try:
                lib.m3r_host_free(self.addr)
            except Exception:
                pass

    # keep the pinned block alive as long as the array (or a view of it) is
    holder = np.ndarray.__new__(_PinnedArray, arr.shape, dtype=arr.dtype, buffer=arr.data)
    holder._owner = _Owner(p)
    return holder


class OutputPool:
    """Recycled page-locked output buffers for the calls that return fresh arrays.

    get(n) returns views of one set of pinned arrays (allocated with `make(n)` when no
    free set of that size exists); once every view of a set -- and every view made from
    them -- has been garbage-collected, the set goes back to the free list (at most
    `keep` free sets per size are kept; the rest are released).  Results the caller
    still holds are never overwritten, and steady-state calls neither allocate host
    memory nor fault fresh pages: copies land directly in page-locked memory.
    """

    def __init__(self, make, keep: int = 2):
        self._make = make
        self._keep = keep
        self._free: dict[int, list] = {}
        self._lock = threading.Lock()

    def get(self, n: int) -> dict:
        import weakref

        with self._lock:
            free = self._free.setdefault(n, [])
            base = free.pop() if free else None
        if base is None:
            base = self._make(n)
        live = [len(base)]

        def _done(_n=n, _base=base, _live=live):
            _live[0] -= 1
            if _live[0] == 0:
                with self._lock:
                    lst = self._free.setdefault(_n, [])
                    if len(lst) < self._keep:
                        lst.append(_base)

        views = {}
        for k, b in base.items():
            # every array handed out (and every view of it) reaches the memory through
            # its lease object, so the lease dies only with the last of them (numpy
            # collapses view chains onto the array that owns the memory, a lease is not one)
            lease = _Lease(b)
            weakref.finalize(lease, _done)
            views[k] = np.frombuffer(lease, dtype=b.dtype).reshape(b.shape)
        return views


class _Lease:
    """Buffer-protocol handle on one pooled array (see OutputPool.get)."""

    def __init__(self, arr: np.ndarray):
        self._arr = arr

    def __buffer__(self, flags):
        return memoryview(self._arr)

    def __release_buffer__(self, view):
        view.release()


class _PinnedArray(np.ndarray):
    _owner = None

    def __array_finalize__(self, obj):
        if obj is not None and getattr(obj, "_owner", None) is not None:
            self._owner = obj._owner
