"""Failure handling of the checkpoint reader on the host (no GPU): m3r_check_checkpoint
runs the same reading and shape checks as m3r_load (the call behind
NativeEngineWrapper.load, native_wrapper.py:57) and turns every malformed file into
M3R_ERR_IO with a message, never a crash: truncated files, a corrupt header, data
offsets past the end of the file, a missing tensor, a wrongly shaped tensor, an
unsupported dtype.  16-bit (F16 / BF16) checkpoints are accepted."""

from __future__ import annotations

import ctypes
import json
import struct

import numpy as np
import pytest

M3R_ERR_IO = -2


@pytest.fixture(scope="module")
def env():
    from mast3r_runtime_b200 import _lib
    from mast3r_runtime_b200._cuda import make_config
    from mast3r_runtime_b200.weights import make_weights, tiny_dims

    d = tiny_dims()
    return _lib.load(), make_config(d, (64, 96)), make_weights(d, seed=2), _lib


def _write(path, tensors: dict, dtype="F32", header_extra=None, raw=None):
    """A safetensors file: 8-byte little-endian header length, JSON header, data."""
    header, blobs, off = {}, [], 0
    for k, v in tensors.items():
        a = np.ascontiguousarray(v, np.float32)
        if dtype == "F16":
            b = a.astype(np.float16).tobytes()
        elif dtype == "BF16":
            b = (a.view(np.uint32) >> 16).astype(np.uint16).tobytes()
        else:
            b = a.tobytes()
        header[k] = {"dtype": dtype, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    if header_extra:
        header.update(header_extra)
    h = json.dumps(header).encode() if raw is None else raw
    path.write_bytes(struct.pack("<Q", len(h)) + h + b"".join(blobs))
    return path


def _check(env, path):
    lib, cfg, _, _lib = env
    rc = lib.m3r_check_checkpoint(ctypes.byref(cfg), str(path).encode())
    return rc, (lib.m3r_global_error() or b"").decode()


def test_valid_checkpoint(env, tmp_path):
    _, _, w, _ = env
    assert _check(env, _write(tmp_path / "ok.safetensors", w)) == (0, "")


@pytest.mark.parametrize("dtype", ["F16", "BF16"])
def test_16bit_checkpoint_accepted(env, tmp_path, dtype):
    _, _, w, _ = env
    assert _check(env, _write(tmp_path / "h.safetensors", w, dtype=dtype))[0] == 0


def test_missing_file(env, tmp_path):
    rc, msg = _check(env, tmp_path / "nope.safetensors")
    assert rc == M3R_ERR_IO and "cannot open" in msg


def test_truncated_file(env, tmp_path):
    _, _, w, _ = env
    p = _write(tmp_path / "t.safetensors", w)
    data = p.read_bytes()
    for cut in (4, 8 + 10, len(data) // 2, len(data) - 1):
        p.write_bytes(data[:cut])
        rc, msg = _check(env, p)
        assert rc == M3R_ERR_IO, (cut, msg)


def test_corrupt_header(env, tmp_path):
    for raw in (b"{not json", b'{"a": {"dtype": "F32", "shape": [2], "data_offsets": [0]}}', b"[]", b"\xff\xfe"):
        rc, msg = _check(env, _write(tmp_path / "c.safetensors", {}, raw=raw))
        assert rc == M3R_ERR_IO, msg


def test_header_length_past_end(env, tmp_path):
    p = tmp_path / "l.safetensors"
    p.write_bytes(struct.pack("<Q", 1 << 40) + b"{}")
    rc, msg = _check(env, p)
    assert rc == M3R_ERR_IO and "header length" in msg


def test_data_offsets_past_end(env, tmp_path):
    _, _, w, _ = env
    bad = {"extra": {"dtype": "F32", "shape": [4], "data_offsets": [0, 1 << 30]}}
    rc, msg = _check(env, _write(tmp_path / "o.safetensors", w, header_extra=bad))
    assert rc == M3R_ERR_IO and "out of file bounds" in msg


def test_missing_tensor(env, tmp_path):
    _, _, w, _ = env
    w2 = {k: v for k, v in w.items() if k != "enc_blocks.1.mlp.fc2.weight"}
    rc, msg = _check(env, _write(tmp_path / "m.safetensors", w2))
    assert rc == M3R_ERR_IO and "missing tensor" in msg and "enc_blocks.1.mlp.fc2.weight" in msg


def test_wrong_shape(env, tmp_path):
    _, _, w, _ = env
    w2 = dict(w)
    w2["dec_blocks.0.attn.qkv.weight"] = w["dec_blocks.0.attn.qkv.weight"][:-1]
    rc, msg = _check(env, _write(tmp_path / "s.safetensors", w2))
    assert rc == M3R_ERR_IO and "has shape" in msg


def test_unsupported_dtype(env, tmp_path):
    _, _, w, _ = env
    p = _write(tmp_path / "d.safetensors", w)
    raw = p.read_bytes()
    hlen = struct.unpack("<Q", raw[:8])[0]
    header = json.loads(raw[8:8 + hlen])
    header["patch_embed.proj.bias"]["dtype"] = "I32"
    h = json.dumps(header).encode()
    p.write_bytes(struct.pack("<Q", len(h)) + h + raw[8 + hlen:])
    rc, msg = _check(env, p)
    assert rc == M3R_ERR_IO and "unsupported dtype" in msg


def test_bad_config_is_an_argument_error(env, tmp_path):
    lib, cfg, w, _lib = env
    bad = _lib.M3RConfig.from_buffer_copy(cfg)
    bad.img_h = 65  # not a multiple of the patch
    rc = lib.m3r_check_checkpoint(ctypes.byref(bad), str(_write(tmp_path / "ok.safetensors", w)).encode())
    assert rc == -1
