"""CPU-side checks of the boundary: the C ABI library loads and exports every function
include/m3r_cuda.h declares, the ctypes layout of m3r_config matches the C compiler's,
the host side behaves like the reference's native-engine contract without a GPU, and the
reference's own NativeEngineWrapper drives CUDAEngine (with a fake device engine)."""

from __future__ import annotations

import ctypes
import re
import subprocess
import sys
import textwrap
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest

from conftest import REFERENCE, ROOT

HEADER = ROOT / "include" / "m3r_cuda.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(m3r_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from mast3r_runtime_b200 import _lib

    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/m3r_cuda.h but not exported"
    # and the ctypes table binds exactly the declared functions
    assert sorted(_lib.SIGNATURES) == names


def declared_prototypes():
    """name -> (return type text, parameter count) of every declaration in the header."""
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    protos = {}
    for ret, name, params in re.findall(r"([A-Za-z_][A-Za-z0-9_ ]*?\**)\s*\b(m3r_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", text):
        params = params.strip()
        n = 0 if params in ("", "void") else params.count(",") + 1
        protos[name] = (ret.split()[-1] if ret.split() else ret, n)
    return protos


def test_ctypes_signatures_match_the_header():
    """Every binding in _lib.SIGNATURES takes as many arguments as its C declaration, and
    the int-returning entry points are bound as returning int."""
    from mast3r_runtime_b200 import _lib

    protos = declared_prototypes()
    assert sorted(protos) == sorted(_lib.SIGNATURES)
    for name, (res, args) in _lib.SIGNATURES.items():
        ret, n = protos[name]
        assert len(args) == n, f"{name}: {len(args)} ctypes arguments, {n} in include/m3r_cuda.h"
        if ret == "int":
            assert res is ctypes.c_int, name
        elif ret == "void":
            assert res is None, name


def test_config_layout_matches_c(tmp_path):
    from mast3r_runtime_b200 import _lib

    src = tmp_path / "layout.c"
    src.write_text(textwrap.dedent("""
        #include <stddef.h>
        #include <stdio.h>
        #include "m3r_cuda.h"
        int main(void) {
          printf("%zu %zu %zu %zu %zu %d %d\\n", sizeof(m3r_config), offsetof(m3r_config, devices),
                 offsetof(m3r_config, max_pairs), offsetof(m3r_config, dtype), offsetof(m3r_config, head),
                 M3R_T_COUNT, M3R_ABI_VERSION);
          return 0;
        }
    """))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", str(HEADER.parent), str(src), "-o", str(exe)], check=True)
    size, off_dev, off_mp, off_dt, off_head, tcount, ver = map(int, subprocess.run(
        [str(exe)], capture_output=True, text=True, check=True).stdout.split())
    C = _lib.M3RConfig
    assert ctypes.sizeof(C) == size
    assert C.devices.offset == off_dev and C.max_pairs.offset == off_mp and C.dtype.offset == off_dt
    assert C.head.offset == off_head
    assert tcount == len(_lib.TIMING_KEYS)
    assert _lib.load().m3r_version() == ver


def test_device_queries_without_gpu_do_not_raise():
    import mast3r_runtime_b200 as m

    assert isinstance(m.is_available(), bool)
    n = m.device_count()
    assert n >= 0


def test_engine_errors_are_exceptions_not_crashes():
    from mast3r_runtime_b200 import NativeEngine, _lib, tiny_dims

    lib = _lib.load()
    n = ctypes.c_int(0)
    lib.m3r_device_count(ctypes.byref(n))
    if n.value > 0:
        pytest.skip("a GPU is visible: this test covers the no-GPU path")
    with pytest.raises(RuntimeError):
        NativeEngine(tiny_dims(), (64, 96), [0], 1)
    # invalid arguments are rejected before any device work
    assert lib.m3r_create(None, None) == -1
    assert b"null" in lib.m3r_global_error()


def test_precision_mapping():
    from mast3r_runtime_b200 import _lib

    assert _lib.dtype_for_precision("fp16") == _lib.DTYPE_F16
    assert _lib.dtype_for_precision("fp32") == _lib.DTYPE_F16
    assert _lib.dtype_for_precision("bf16") == _lib.DTYPE_BF16
    with pytest.raises(ValueError):
        _lib.dtype_for_precision("int4")


def test_cuda_engine_construction_and_state():
    from mast3r_runtime_b200 import CUDAEngine

    with pytest.raises(RuntimeError):
        CUDAEngine(variant="no_such_variant")
    with pytest.raises(RuntimeError):
        CUDAEngine(variant="mast3r_vit_large", resolution=500)  # not a multiple of 16
    e = CUDAEngine(variant="mast3r_vit_large", resolution=512, precision="fp16")
    assert not e.is_ready()
    with pytest.raises(RuntimeError):
        e.infer(np.zeros((512, 512, 3), np.uint8), np.zeros((512, 512, 3), np.uint8))
    with pytest.raises(RuntimeError):
        e.load("/nonexistent/unified.safetensors")


def test_weight_shapes_cover_reference_keys():
    from mast3r_runtime_b200.weights import VARIANTS, weight_shapes

    s = weight_shapes(VARIANTS["mast3r_vit_large"])
    assert s["patch_embed.proj.weight"] == (1024, 3, 16, 16)
    assert s["enc_blocks.23.attn.qkv.weight"] == (3072, 1024)
    assert s["dec_blocks2.11.cross_attn.projv.weight"] == (768, 768)
    assert s["downstream_head2.head_local_features.fc2.weight"] == (25 * 256, 7168)
    assert s["downstream_head1.dpt.act_postprocess.0.1.weight"] == (96, 96, 4, 4)
    n = sum(int(np.prod(v)) for v in s.values())
    assert 600e6 < n < 750e6


def test_flops_per_pair_vit_large():
    sys.path.insert(0, str(ROOT))
    import bench
    from mast3r_runtime_b200.weights import VARIANTS

    f = bench.flops_per_pair(VARIANTS["mast3r_vit_large"], (384, 512))
    assert 1.75e12 < f < 1.95e12  # 1.87 TFLOP per pair (two views), 2 FLOP per multiply-add


class FakeNative:
    """Stands in for the device engine: shapes and types of the real one, zeros inside."""

    def __init__(self, dims, hw, devices, max_pairs, dtype):
        self.dims, self.image_hw, self.dtype = dims, tuple(hw), dtype
        self.loaded = None

    def load(self, path):
        self.loaded = path

    def is_ready(self):
        return self.loaded is not None

    def infer_batch(self, img1, img2, out=None):
        n = img1.shape[0]
        H, W = self.image_hw
        o = {"pts3d_1": np.zeros((n, H, W, 3), np.float32), "pts3d_2": np.zeros((n, H, W, 3), np.float32),
             "desc_1": np.zeros((n, H, W, 24), np.float32), "desc_2": np.zeros((n, H, W, 24), np.float32),
             "conf_1": np.ones((n, H, W), np.float32), "conf_2": np.ones((n, H, W), np.float32)}
        return o, {"inference_ms": 1.0, "total_ms": 2.0}

    def match(self, d1, d2, top_k=512, reciprocal=True, confidence_threshold=0.5, conf_1=None, conf_2=None,
              pts3d_1=None, pts3d_2=None):
        k = 3
        return SimpleNamespace(idx_1=np.arange(k, dtype=np.int64), idx_2=np.arange(k, dtype=np.int64),
                               pts2d_1=np.zeros((k, 2), np.float32), pts2d_2=np.zeros((k, 2), np.float32),
                               pts3d_1=np.zeros((k, 3), np.float32), pts3d_2=np.zeros((k, 3), np.float32),
                               confidence=np.ones(k, np.float32), timing={"match_ms": 0.1})

    def close(self):
        pass


def test_reference_wrapper_drives_cuda_engine(monkeypatch, tmp_path):
    if REFERENCE is None or not (REFERENCE / "mast3r_runtime").is_dir():
        pytest.skip("reference tree not present")
    sys.dont_write_bytecode = True
    sys.path.insert(0, str(REFERENCE))
    import mast3r_runtime_b200
    from mast3r_runtime_b200 import _cuda

    monkeypatch.setattr(_cuda, "NativeEngine", FakeNative)
    mast3r_runtime_b200.install()
    from mast3r_runtime.backends import get_available_backends, get_runtime
    from mast3r_runtime.backends.native_wrapper import NativeEngineWrapper
    from mast3r_runtime.core.config import BackendType, MASt3RRuntimeConfig, ModelConfig, RuntimeConfig

    cfg = MASt3RRuntimeConfig(model=ModelConfig(resolution=336), runtime=RuntimeConfig(backend=BackendType.CUDA),
                              cache_dir=tmp_path)
    # the weights file where get_default_model_path puts it (core/config.py:477-505)
    wpath = tmp_path / "safetensors" / "dune_vit_small_336" / "decoder.safetensors"
    wpath.parent.mkdir(parents=True)
    wpath.write_bytes(b"\0" * 16)
    assert isinstance(get_available_backends()["cuda"], bool)
    engine = get_runtime(cfg)
    assert isinstance(engine, NativeEngineWrapper)
    engine.load()
    assert engine.is_ready
    img = np.zeros((336, 336, 3), np.uint8)
    res = engine.infer(img, img)
    assert res.pts3d_1.shape == (336, 336, 3) and res.desc_1.shape == (336, 336, 24) and res.conf_2.shape == (336, 336)
    assert res.timing_ms["inference_ms"] == 1.0
    m = engine.match(res.desc_1, res.desc_2)
    assert m.num_matches == 3 and m.idx_1.dtype == np.int64
    sys.modules.pop("mast3r_runtime.backends._cuda", None)


def test_output_pool_recycles_only_released_sets():
    """OutputPool (pinned outputs of the drop-in calls): a set comes back only when every
    view of it -- including views made from the returned arrays -- is gone."""
    import gc

    from mast3r_runtime_b200 import _lib

    made = []

    def make(n):
        d = {"a": np.zeros((n, 4), np.float32), "b": np.zeros((n, 2), np.float32)}
        made.append(d)
        return d

    pool = _lib.OutputPool(make, keep=1)
    v1 = pool.get(3)
    v1["a"][:] = 1
    inner = v1["a"][0]          # a view of a view keeps the set in use
    del v1
    gc.collect()
    v2 = pool.get(3)            # first set still referenced through `inner`
    assert len(made) == 2 and np.all(inner == 1)
    del inner, v2
    gc.collect()
    v3 = pool.get(3)            # a released set is reused (keep=1: one stays on the free list)
    assert len(made) == 2
    assert v3["a"].base is not None
    v4 = pool.get(5)            # another size: a new set
    assert len(made) == 3 and v4["a"].shape == (5, 4)
