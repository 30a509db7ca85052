"""B200-native (sm_100a) CUDA backend for mast3r-runtime's two-view inference path.

    from mast3r_runtime_b200 import CUDAEngine, install
    install()   # BackendType.CUDA now selects this backend in the reference package

The compute runs in libm3r_cuda.so (hand-written tcgen05 / TMA kernels) behind the
C ABI declared in include/m3r_cuda.h; this package is its ctypes host side.
"""

from ._cuda import (  # noqa: F401
    CUDAEngine,
    NativeEngine,
    device_count,
    get_compute_capability,
    get_device_name,
    install,
    is_available,
)
from .weights import VARIANTS, ModelDims, make_weights, save_safetensors, tiny_dims, weight_shapes  # noqa: F401

__all__ = [
    "CUDAEngine", "NativeEngine", "install", "is_available", "device_count", "get_device_name",
    "get_compute_capability", "VARIANTS", "ModelDims", "make_weights", "save_safetensors", "tiny_dims",
    "weight_shapes",
]
