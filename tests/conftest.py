"""Shared fixtures.  Tests marked ``gpu`` need a B200 and call the CUDA path through the
C ABI; everything else runs on the CPU (oracle vs golden vectors, ABI surface, host logic)."""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = ROOT / "tests" / "golden"
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(GOLDEN))

# the reference tree, when a test may read it (M3R_REFERENCE); tests that need it skip without it
REFERENCE = Path(os.environ["M3R_REFERENCE"]) if os.environ.get("M3R_REFERENCE") else None


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libm3r_cuda.so")


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit pattern (uint16), round to nearest even."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return r.astype(np.uint16)


def from_bf16_bits(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    return from_bf16_bits(to_bf16_bits(x))


DTYPES = {"fp16": 1, "bf16": 0}  # M3R_DTYPE_F16 / M3R_DTYPE_BF16


def to16(x: np.ndarray, dtype: str) -> np.ndarray:
    """float32 -> 16-bit operand bits of `dtype` ("fp16" or "bf16"), round to nearest even."""
    if dtype == "fp16":
        return np.ascontiguousarray(x, np.float32).astype(np.float16).view(np.uint16)
    return to_bf16_bits(x)


def from16(b: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "fp16":
        return b.view(np.float16).astype(np.float32)
    return from_bf16_bits(b)


def round16(x: np.ndarray, dtype: str) -> np.ndarray:
    return from16(to16(x, dtype), dtype)


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def matcher_inputs(h, w, d, seed, dup_frac=0.3, sigma=0.05):
    """Set B: `dup_frac` of its rows are noisy copies of set-A rows, the rest fresh Gaussian."""
    rng = np.random.default_rng(seed)
    n = h * w
    a = rng.standard_normal((n, d)).astype(np.float32)
    b = rng.standard_normal((n, d)).astype(np.float32)
    m = int(dup_frac * n)
    dst = rng.permutation(n)[:m]
    src = rng.permutation(n)[:m]
    b[dst] = a[src] + np.float32(sigma) * rng.standard_normal((m, d)).astype(np.float32)
    return a.reshape(h, w, d), b.reshape(h, w, d)


@pytest.fixture(scope="session")
def oracle_lib():
    import oracle

    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def have_reference():
    return REFERENCE is not None and (REFERENCE / "mast3r_runtime").is_dir()
