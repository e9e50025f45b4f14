"""Parity of the SDXL UNet step and VAE decoder against the numpy oracle (oracle/sdxl.py) at reduced widths
(the same kernels and block structure as the full model; the full sizes run in bench.py).

Bars: the reference's own (tests/sdxl_ref_test.cpp:242, 301): UNet pass rel-RMS < 0.02, VAE rel-RMS < 0.01; plus a
cosine >= 0.999 on every probed stage."""

import numpy as np
import pytest

from oracle import rng
from oracle import sdxl as OS

pytestmark = pytest.mark.gpu


def _cos(a, b):
    a, b = a.astype(np.float64).ravel(), b.astype(np.float64).ravel()
    return float(a @ b / np.sqrt((a @ a) * (b @ b)))


def _rel(a, b):
    a, b = a.astype(np.float64), b.astype(np.float64)
    return float(np.sqrt(((a - b) ** 2).sum() / (b ** 2).sum()))


def test_unet_step_reduced(cuda):
    import mkimage

    cfg = dict(channels=(64, 128, 256), depth=(0, 1, 2), layers=2, context_dim=256, pooled_dim=128)
    gh, gw, S, B = 16, 16, 77, 2
    u = mkimage.Unet(mkimage.UnetConfig(max_batch=B, max_gh=gh, max_gw=gw, max_context=S, slots=2, **cfg))
    u.init_random(17)
    W = u.weights()
    oc = OS.unet_default_cfg(**cfg)
    ctxs = [rng.normal(rng.tensor_key(3, 10 + b), S * 256).reshape(S, 256) for b in range(B)]
    pooled = [rng.normal(rng.tensor_key(3, 20 + b), 128) for b in range(B)]
    lats = np.stack([rng.normal(rng.tensor_key(3, 30 + b), gh * gw * 16).reshape(gh * gw, 16) * 3.0
                     for b in range(B)])
    sigmas = [2.5, 7.0]
    for b in range(B):
        u.begin(ctxs[b], pooled[b], gh, gw, slot=b)
    got = {}
    u.set_probe(lambda name, layer, a: got.__setitem__(name, a))
    eps = u.step_batch(lats, sigmas)
    u.set_probe(None)
    for b in range(B):
        st = OS.unet_begin(oc, W, ctxs[b], pooled[b], gh, gw)
        want = {}
        ref = OS.unet_step(oc, W, st, lats[b], sigmas[b], probe=lambda n, a: want.__setitem__(n, a))
        for name in ("conv_in", "in1.res", "in3.down", "in4.attn", "in8.attn", "mid.attn", "out0.attn", "out2.up",
                     "out8.res"):
            g = got[name].reshape(B, -1)[b]
            w = want[name].ravel()
            assert _cos(g, w) >= 0.999, (name, _cos(g, w))
        assert _rel(eps[b], ref) < 0.02 and _cos(eps[b], ref) >= 0.999, (_rel(eps[b], ref), _cos(eps[b], ref))
    # the graph-replayed step (third call) equals the eager one
    e2 = u.step_batch(lats, sigmas)
    e3 = u.step_batch(lats, sigmas)
    assert np.array_equal(e2, eps) and np.array_equal(e3, eps)
    # a single step on slot 1 matches that sample of the batch
    e1 = u.step(lats[1], sigmas[1], slot=1)
    assert np.abs(e1 - eps[1]).max() <= 1e-5 * max(1.0, np.abs(eps[1]).max())


def test_unet_geglu_bias_order(cuda):
    """The GEGLU projection's bias follows its rows into the interleaved device layout: with unit-scale ff1 biases
    (the random init's 0.02 hides a misplaced bias) the step still matches the oracle."""
    import mkimage

    cfg = dict(channels=(64, 128, 256), depth=(0, 1, 2), layers=1, context_dim=256, pooled_dim=128)
    gh, gw, S = 8, 16, 77
    u = mkimage.Unet(mkimage.UnetConfig(max_batch=1, max_gh=gh, max_gw=gw, max_context=S, slots=1, **cfg))
    u.init_random(19)
    for i, (name, shape) in enumerate(u.weight_names()):
        if name.endswith(".ff1.b"):
            u.write_weight(name, rng.normal(rng.tensor_key(6, i), shape[0]))
    W = u.weights()
    ctx = rng.normal(rng.tensor_key(6, 1000), S * 256).reshape(S, 256)
    pooled = rng.normal(rng.tensor_key(6, 1001), 128)
    lat = rng.normal(rng.tensor_key(6, 1002), gh * gw * 16).reshape(gh * gw, 16)
    u.begin(ctx, pooled, gh, gw, slot=0)
    eps = u.step(lat, 3.0, slot=0)
    oc = OS.unet_default_cfg(**cfg)
    ref = OS.unet_step(oc, W, OS.unet_begin(oc, W, ctx, pooled, gh, gw), lat, 3.0)
    assert _rel(eps, ref) < 0.02 and _cos(eps, ref) >= 0.999, (_rel(eps, ref), _cos(eps, ref))


def test_vae_decode_reduced(cuda):
    _vae_reduced_check()


def _vae_reduced_check():
    """The decoder at channels 128/128/256/256 (GroupNorm groups of 4 and 8 channels), one layer, an 8 x 8 latent."""
    import mkimage

    cfg = dict(channels=(128, 128, 256, 256), layers=1)
    gh, gw = 8, 8
    v = mkimage.Vae(mkimage.VaeConfig(max_gh=gh, max_gw=gw, **cfg))
    v.init_random(23)
    W = v.weights()
    lat = rng.normal(rng.tensor_key(4, 1), gh * gw * 16).reshape(gh * gw, 16) * 0.13025
    got = {}
    v.set_probe(lambda name, layer, a: got.__setitem__(name, a))
    img = v.decode(lat, gh, gw)
    v.set_probe(None)
    want = {}
    ref = OS.vae_decode(OS.vae_default_cfg(**cfg), W, lat, gh, gw, probe=lambda n, a: want.__setitem__(n, a))
    for name in ("mid.attn", "mid.res1", "up0.up", "up3.res1"):
        assert _cos(got[name], want[name].ravel()) >= 0.999, name
    assert img.shape == (128, 128, 4) and np.all(img[..., 3] == 1.0)
    assert _rel(img, ref) < 0.01, _rel(img, ref)


_THREE_PASS_CHILD = r"""
import sys
sys.path[:0] = [{root!r}, {pkg!r}]
from tests.test_sdxl_gpu import _vae_reduced_check
_vae_reduced_check()
print("THREE_PASS_OK")
"""


def test_vae_decode_three_pass_group_norm(cuda):
    """The decode above with every GroupNorm taking its statistics in a pass of its own (MKB_GN_FUSED=0) instead of
    from the convolution that wrote its input. The switch is read once per process, so this runs in a child."""
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = _THREE_PASS_CHILD.format(root=root, pkg=os.path.join(root, "mako-image_b200"))
    r = subprocess.run([sys.executable, "-c", code], env=dict(os.environ, MKB_GN_FUSED="0"), capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0 and "THREE_PASS_OK" in r.stdout, (r.stdout[-2000:], r.stderr[-4000:])


def test_vae_decode_16_latent_channels(cuda):
    """The decoder of a 16-channel latent (tokens of 64 values, the DiT's) with per-value latent statistics."""
    import mkimage

    cfg = dict(channels=(128, 128, 128, 256), layers=1, latent=16)
    gh, gw = 4, 8
    v = mkimage.Vae(mkimage.VaeConfig(max_gh=gh, max_gw=gw, **cfg))
    v.init_random(29)
    mean = (0.3 * rng.normal(rng.tensor_key(4, 5), 64)).astype(np.float32)
    std = (1.0 + 0.5 * np.abs(rng.normal(rng.tensor_key(4, 6), 64))).astype(np.float32)
    v.set_latent_stats(mean, std)
    W = v.weights()
    lat = rng.normal(rng.tensor_key(4, 7), gh * gw * 64).reshape(gh * gw, 64)
    img = v.decode(lat, gh, gw)
    ref = OS.vae_decode(OS.vae_default_cfg(**cfg), W, lat, gh, gw, stats=(mean, std))
    assert img.shape == (16 * gh, 16 * gw, 4)
    assert _rel(img, ref) < 0.01 and _cos(img, ref) >= 0.999, (_rel(img, ref), _cos(img, ref))


def test_sdxl_schedule():
    import mkimage

    s = mkimage.sdxl_sigmas(28)
    assert s.shape == (29,) and s[-1] == 0 and np.all(np.diff(s[:-1]) < 0)
    assert abs(s[0] - 14.6146) < 1e-3  # sigma at t = 999 of the scaled-linear schedule
    table = OS.discrete_log_sigmas()
    for sg in (0.03, 1.0, 5.5, 14.6):
        assert mkimage.sdxl_timestep(sg) == OS.timestep(sg)
    assert np.allclose(np.log(s[[0, 27]]), table[[999, 0]], atol=1e-5)
