"""The FMA-pipe exponential of the attention softmax (exp2_poly2 in
mast3r_runtime_b200/csrc/attention.cu), restated in numpy float32 arithmetic with the
constants read from the kernel source: the 16-bit pattern of 2^(v + 0.5) is built as
round(2^m (v + 0.5 + e + g)) in the low bits of an fp32 word (Schraudolph's bit-pattern
exponential with a minimax cubic correction g after a round-to-nearest range reduction).

Bound: within 0.62 ulp of the fp16 result over the normal range (round to nearest
is 0.5 ulp), 0.52 ulp of bf16; results below the smallest normal fp16 are within
4e-5 absolute (the row maximum contributes 1)."""

from __future__ import annotations

import re

import numpy as np

from conftest import ROOT

SRC = (ROOT / "mast3r_runtime_b200" / "csrc" / "attention.cu").read_text()


def _const(name: str) -> np.float32:
    m = re.search(rf"\b{name}\s*=\s*([-0-9.eE]+)f", SRC)
    assert m, name
    return np.float32(float(m.group(1)))


def _fma(a, b, c):
    # a * b is exact in float64 for float32 inputs; one rounding of the sum to float32
    return (np.asarray(a, np.float64) * np.asarray(b, np.float64) + np.asarray(c, np.float64)).astype(np.float32)


def _poly_bits(v, scale, bias, vmin):
    f32 = np.float32
    sh = _const("kShifter")
    g = [_const(f"kG{i}") for i in range(4)]
    v = np.fmax(np.asarray(v, f32), f32(vmin))  # fmaxf: a NaN operand gives the other
    n = ((v + sh).astype(f32) - sh).astype(f32)
    f = (v - n).astype(f32)
    q = _fma(f, g[3], g[2])
    q = _fma(q, f, g[1])
    q = _fma(q, f, g[0])
    t = (v + q).astype(f32)
    y = _fma(t, f32(scale), f32(float(sh) + scale * bias))
    return (y.view(np.uint32) & 0xFFFF).astype(np.uint16)


def test_constants_present():
    assert float(_const("kShifter")) == 1.5 * 2 ** 23


def test_fp16_pattern_accuracy():
    v = np.linspace(-20.0, 8.0, 1_000_001, dtype=np.float32)
    h = _poly_bits(v, 1024.0, 15.5, -15.5)
    got = h.view(np.float16).astype(np.float64)
    want = np.exp2(v.astype(np.float64) + 0.5)
    normal = want >= 2.0 ** -14
    ulp = 2.0 ** (np.floor(np.log2(want[normal])) - 10)
    assert (np.abs(got[normal] - want[normal]) / ulp).max() <= 0.62
    assert np.abs(got[~normal] - want[~normal]).max() <= 4e-5
    assert np.all(np.isfinite(got)) and np.all(got >= 0)


def test_bf16_pattern_accuracy():
    v = np.linspace(-70.0, 8.0, 1_000_001, dtype=np.float32)
    h = _poly_bits(v, 128.0, 127.5, -60.0)
    got = (h.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    want = np.exp2(v.astype(np.float64) + 0.5)
    ok = v >= -60.0
    ulp = 2.0 ** (np.floor(np.log2(want[ok])) - 7)
    assert (np.abs(got[ok] - want[ok]) / ulp).max() <= 0.52
    assert np.abs(got[~ok]).max() <= 2.0 ** -59


def test_masked_scores_give_zero():
    h = _poly_bits(np.array([-np.inf, -1e30, np.nan], np.float32), 1024.0, 15.5, -15.5)
    assert np.all(h.view(np.float16) == 0)
