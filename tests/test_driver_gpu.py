"""The mako_image driver (mako-image_b200/bin/mako_image): seeded random models, a few denoising steps, VAE decode,
PNG out. The PNG must read back (tests/test_png_cpu.py's reader: chunk CRCs, zlib stream), carry the provenance
text chunks the reference writes, and hold exactly the 8-bit image that the VAE makes of the run's final latents
(decoded again here through the Python binding with the same seeded weights); a second run of the same seed must
write the same bytes."""

import json
import os
import subprocess

import numpy as np
import pytest

from tests.test_png_cpu import read_png

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "mako-image_b200", "bin", "mako_image")
VAE = ["--vae-channels", "128,128,128,128", "--vae-layers", "1"]


def _run(args, tmp_path, name):
    png, lat = tmp_path / f"{name}.png", tmp_path / f"{name}.f32"
    r = subprocess.run([BIN, *args, "-o", str(png), "--latents-out", str(lat)], capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    return png.read_bytes(), np.fromfile(lat, np.float32)


def _decode_again(latent, scale, lat, gh, gw):
    import mkimage

    v = mkimage.Vae(mkimage.VaeConfig(channels=(128, 128, 128, 128), layers=1, latent=latent, scale=scale,
                                      max_gh=gh, max_gw=gw))
    v.init_random(2)  # the driver's VAE seed: --weights-seed (1) + 1
    img = v.decode(lat.reshape(gh * gw, 4 * latent), gh, gw)
    v.close()
    out = np.empty(img.size, np.uint8)
    import ctypes

    mkimage.check(mkimage.lib.mkb_to_rgba8(img.ctypes.data_as(ctypes.c_void_p), img.size,
                                           out.ctypes.data_as(ctypes.c_void_p)))
    return out.reshape(img.shape)


@pytest.mark.parametrize("model", ["qwen", "sdxl"])
def test_driver_writes_the_decoded_image(cuda, tmp_path, model):
    if not os.path.exists(BIN):
        subprocess.run(["make", "-C", os.path.join(ROOT, "mako-image_b200"), "-s"], check=True)
    size = 256
    common = ["random", "a lighthouse at dusk", "--model", model, "--width", str(size), "--height", str(size),
              "--steps", "3", "--seed", "7", "--guidance", "3.5", *VAE]
    if model == "qwen":
        common += ["--dims", "256,2,512,2,128"]
    else:
        common += ["--unet-channels", "64,128,256", "--unet-depth", "0,1,1"]
    data, lat = _run(common, tmp_path, "a")
    w, h, ctype, px, text = read_png(data)
    assert (w, h, ctype) == (size, size, 6)
    assert np.all(px[..., 3] == 255)
    assert np.isfinite(lat).all() and lat.std() > 0
    latent = 16 if model == "qwen" else 4
    gh = gw = size // 16
    assert lat.size == gh * gw * 4 * latent
    want = _decode_again(latent, 1.0 if model == "qwen" else 0.13025, lat, gh, gw)
    assert np.array_equal(px, want)
    assert px[..., :3].std() > 0  # not a constant image
    # Provenance, as the reference's with_provenance writes it.
    params = text["parameters"].split("\n")
    assert params[0] == "a lighthouse at dusk"
    assert params[1] == "Negative prompt: (embeddings)"
    assert params[2] == f"Steps: 3, Sampler: Euler, CFG scale: 3.5, Seed: 7, Size: {size}x{size}, Model: random-{model}"
    meta = json.loads(text["mako"])
    assert meta["steps"] == 3 and meta["seed"] == 7 and meta["sampler"] == "euler" and meta["guidance"] == 3.5
    assert meta["width"] == size and meta["loras"] == []
    # Same seed, same bytes.
    data2, _ = _run(common, tmp_path, "b")
    assert data2 == data


def test_driver_rejects_bad_arguments(cuda, tmp_path):
    r = subprocess.run([BIN, "random", "x", "--width", "100"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 1 and "multiples of 16" in r.stderr
    r = subprocess.run([BIN, "random", "x", "--sampler", "ddim"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 1 and "sampler" in r.stderr
