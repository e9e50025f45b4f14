"""The library's PNG writer and 8-bit conversion (mkb_png_encode, mkb_to_rgba8), read back with Python's zlib: chunk
CRCs, the IHDR fields, and the decompressed scanlines equal to the input samples, for RGBA and RGB, across the
65535-byte stored-block boundary. No device is needed."""

import ctypes
import struct
import zlib

import numpy as np
import pytest


def _encode(mk, rgba8, rgb=False):
    h, w, _ = rgba8.shape
    a = np.ascontiguousarray(rgba8, np.uint8)
    size = ctypes.c_size_t()
    mk.check(mk.lib.mkb_png_encode(a.ctypes.data_as(ctypes.c_void_p), w, h, int(rgb), None, 0, ctypes.byref(size)))
    out = (ctypes.c_uint8 * size.value)()
    mk.check(mk.lib.mkb_png_encode(a.ctypes.data_as(ctypes.c_void_p), w, h, int(rgb), out, size.value,
                                   ctypes.byref(size)))
    return bytes(out)


def read_png(data):
    """(width, height, colour type, samples [h][w][c], {text keyword: text}) of an 8-bit PNG with filter-0 rows."""
    assert data[:8] == b"\x89PNG\r\n\x1a\n"
    i, idat, text, ihdr = 8, b"", {}, None
    while i < len(data):
        n, = struct.unpack(">I", data[i:i + 4])
        typ, body = data[i + 4:i + 8], data[i + 8:i + 8 + n]
        crc, = struct.unpack(">I", data[i + 8 + n:i + 12 + n])
        assert crc == zlib.crc32(typ + body) & 0xFFFFFFFF, typ
        if typ == b"IHDR":
            ihdr = struct.unpack(">IIBBBBB", body)
        elif typ == b"IDAT":
            idat += body
        elif typ == b"iTXt":
            key, rest = body.split(b"\0", 1)
            assert rest[:2] == b"\0\0"
            _, rest = rest[2:].split(b"\0", 1)  # language tag
            _, txt = rest.split(b"\0", 1)       # translated keyword
            text[key.decode()] = txt.decode("utf-8")
        i += 12 + n
        if typ == b"IEND":
            assert i == len(data)
    w, h, depth, ctype, comp, filt, inter = ihdr
    assert depth == 8 and comp == 0 and filt == 0 and inter == 0
    c = {6: 4, 2: 3}[ctype]
    raw = np.frombuffer(zlib.decompress(idat), np.uint8).reshape(h, 1 + w * c)
    assert np.all(raw[:, 0] == 0)
    return w, h, ctype, raw[:, 1:].reshape(h, w, c), text


@pytest.mark.parametrize("h,w", [(1, 1), (23, 37), (200, 300)])
@pytest.mark.parametrize("rgb", [False, True])
def test_png_roundtrip(h, w, rgb):
    import mkimage

    img = np.random.RandomState(h * w).randint(0, 256, (h, w, 4)).astype(np.uint8)
    pw, ph, ctype, px, _ = read_png(_encode(mkimage, img, rgb))
    assert (pw, ph, ctype) == (w, h, 2 if rgb else 6)
    assert np.array_equal(px, img[..., :3] if rgb else img)


def test_png_rejects_small_buffer():
    import mkimage

    img = np.zeros((4, 4, 4), np.uint8)
    size = ctypes.c_size_t()
    out = (ctypes.c_uint8 * 8)()
    code = mkimage.lib.mkb_png_encode(img.ctypes.data_as(ctypes.c_void_p), 4, 4, 0, out, 8, ctypes.byref(size))
    assert code == 1 and size.value > 8


def test_to_rgba8():
    import mkimage

    x = np.concatenate([np.linspace(-1.5, 1.5, 1001, dtype=np.float32),
                        (np.arange(256, dtype=np.float32) + 0.5) / 127.5 - 1.0]).astype(np.float32)  # half-way points
    out = np.empty(x.size, np.uint8)
    mkimage.check(mkimage.lib.mkb_to_rgba8(x.ctypes.data_as(ctypes.c_void_p), x.size,
                                           out.ctypes.data_as(ctypes.c_void_p)))
    v = np.clip(x * np.float32(0.5) + np.float32(0.5), 0, 1).astype(np.float32) * np.float32(255.0)
    assert np.array_equal(out, np.rint(v).astype(np.uint8))
