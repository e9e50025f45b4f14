"""The safetensors reader (mkb_st_*) on the CPU: values of F32 / F16 / BF16 files written by an independent writer
(tests/st_files.py), F16 special values, metadata and names, and malformed files rejected with an error."""

import json
import os
import struct
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "mako-image_b200"))

from st_files import bf16_value, write_safetensors  # noqa: E402


def test_reader_values_all_dtypes(tmp_path):
    import mkimage

    rng = np.random.RandomState(3)
    a = rng.standard_normal((7, 13)).astype(np.float32) * 10
    b = rng.standard_normal((5,)).astype(np.float32)
    c = rng.standard_normal((2, 3, 4)).astype(np.float32)
    p = tmp_path / "m.safetensors"
    write_safetensors(p, {"a.weight": (a, "F32"), "b.bias": (b, "F16"), "c": (c, "BF16"), "empty": (np.zeros(0), "F32"),
                          "blk.é": (b, "F32")}, metadata={"format": "pt"})
    got = mkimage.st_read(p)
    assert set(got) == {"a.weight", "b.bias", "c", "empty", "blk.é"}
    assert got["a.weight"][0] == "F32" and np.array_equal(got["a.weight"][1], a)
    assert got["b.bias"][0] == "F16" and np.array_equal(got["b.bias"][1], b.astype(np.float16).astype(np.float32))
    assert got["c"][0] == "BF16" and np.array_equal(got["c"][1], bf16_value(c).reshape(c.shape))
    assert got["empty"][1].shape == (0,)


def test_reader_f16_special_values(tmp_path):
    import mkimage

    bits = np.array([0x0000, 0x8000, 0x0001, 0x03FF, 0x0400, 0x7BFF, 0x7C00, 0xFC00, 0x3C00, 0xC000, 0x0200],
                    np.uint16)
    vals = bits.view(np.float16).astype(np.float32)
    p = tmp_path / "h.safetensors"
    write_safetensors(p, {"h": (vals, "F16")})
    got = mkimage.st_read(p)["h"][1]
    assert np.array_equal(got.view(np.uint32), vals.view(np.uint32))  # bit-exact, signed zero included
    nanbits = np.array([0x7E00], np.uint16).view(np.float16).astype(np.float32)
    write_safetensors(p, {"n": (nanbits, "F16")})
    assert np.isnan(mkimage.st_read(p)["n"][1]).all()


def _raw(path, header, data=b"", hlen=None):
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h) if hlen is None else hlen))
        f.write(h)
        f.write(data)


@pytest.mark.parametrize("case", ["short", "hlen", "json", "offsets", "size", "shape", "overflow", "dtype_read",
                                  "dup_ok"])
def test_reader_rejects_malformed(tmp_path, case):
    import mkimage

    p = tmp_path / "bad.safetensors"
    ok = {"t": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]}}
    if case == "short":
        p.write_bytes(b"\x01\x02")
    elif case == "hlen":
        _raw(p, ok, b"\0" * 8, hlen=1 << 40)
    elif case == "json":
        with open(p, "wb") as f:
            f.write(struct.pack("<Q", 5) + b'{"t":')
    elif case == "offsets":
        _raw(p, {"t": {"dtype": "F32", "shape": [2], "data_offsets": [0, 64]}}, b"\0" * 8)
    elif case == "size":
        _raw(p, {"t": {"dtype": "F32", "shape": [3], "data_offsets": [0, 8]}}, b"\0" * 8)
    elif case == "shape":
        _raw(p, {"t": {"dtype": "F32", "shape": [-2], "data_offsets": [0, 8]}}, b"\0" * 8)
    elif case == "overflow":  # 2^32 x 2^32 elements: the 64-bit product wraps to 0, which would match [0, 0)
        _raw(p, {"t": {"dtype": "F32", "shape": [1 << 32, 1 << 32], "data_offsets": [0, 0]}})
        with pytest.raises(mkimage.MkbError, match="too large"):
            mkimage.st_read(p)
        return
    elif case == "dtype_read":
        _raw(p, {"t": {"dtype": "I64", "shape": [1], "data_offsets": [0, 8]}}, b"\0" * 8)
        with pytest.raises(mkimage.MkbError, match="unsupported dtype"):
            mkimage.st_read(p)
        return
    elif case == "dup_ok":  # a valid file for contrast
        _raw(p, ok, struct.pack("<2f", 1.5, -2.0))
        assert np.array_equal(mkimage.st_read(p)["t"][1], np.array([1.5, -2.0], np.float32))
        return
    with pytest.raises(mkimage.MkbError):
        mkimage.st_read(p)
