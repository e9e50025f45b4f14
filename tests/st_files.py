"""A safetensors writer for the tests (independent of the library's reader, which the tests check against it).

Layout: an 8-byte little-endian header length, a JSON header {name: {dtype, shape, data_offsets}, __metadata__},
then the raw little-endian tensor bytes in header order."""

import json
import struct

import numpy as np


def bf16_bits(a):
    """float32 -> bfloat16 bit patterns, round to nearest even (NaN kept NaN)."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(a, np.float32))
    r[nan] = 0x7FC0
    return r


def bf16_value(a):
    """The float32 values bf16_bits encodes."""
    return (bf16_bits(a).astype(np.uint32) << 16).view(np.float32)


def encode(a, dtype):
    a = np.asarray(a, np.float32)
    if dtype == "F32":
        return a.astype("<f4").tobytes()
    if dtype == "F16":
        return a.astype("<f2").tobytes()
    if dtype == "BF16":
        return bf16_bits(a).astype("<u2").tobytes()
    raise ValueError(dtype)


def write_safetensors(path, tensors, metadata=None, dtype="F32"):
    """tensors: {name: array} or {name: (array, dtype)}; returns the header dict written."""
    header, blobs, off = {}, [], 0
    for name, v in tensors.items():
        a, dt = v if isinstance(v, tuple) else (v, dtype)
        a = np.asarray(a, np.float32)
        b = encode(a, dt)
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    if metadata:
        header["__metadata__"] = metadata
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)
    return header
