"""Parity at the widths and lengths of the benchmark configurations, which the other tests reach only at reduced
sizes: the full-width SDXL UNet (channels 320/640/1280, transformer depths 0/2/10, 5/10/20 heads of 64, a 77 x 2048
context) and VAE decoder (128/256/512/512, two layers per level, the d=512 mid attention) on small canvases the
numpy oracle finishes in seconds, head-dim-128 attention at the 1024^2 (4352 keys) and 2048^2 (17408 keys) joint
lengths, head-dim-64 attention with 20 heads over 1024 keys, and the projections and convolutions of the UNet's
1280-channel level at their 1024^2 sizes.

Bars: the reference's own for whole passes (tests/sdxl_ref_test.cpp:242, 301: UNet rel-RMS < 0.02, VAE < 0.01),
cosine >= 0.999 on every probed stage; attention max-abs <= 2e-2 and cosine >= 0.999 (bf16 P and outputs); fp32
projections within 1e-3 of the output scale. This file sorts after the other kernel tests, so a failure here does
not hide theirs."""

import numpy as np
import pytest

from oracle import ops as O
from oracle import rng
from oracle import sdxl as OS

pytestmark = pytest.mark.gpu


def _cos(a, b):
    a, b = np.asarray(a, np.float64).ravel(), np.asarray(b, np.float64).ravel()
    return float(a @ b / np.sqrt((a @ a) * (b @ b)))


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.sqrt(((a - b) ** 2).sum() / (b ** 2).sum()))


def _np(t):
    return t.float().cpu().numpy()


def _randn(shape, seed, scale=1.0, dev=None, dtype=None):
    import torch

    g = torch.Generator().manual_seed(seed)
    t = torch.randn(*shape, generator=g) * scale
    if dtype is not None:
        t = t.to(dtype)
    return t.to(dev) if dev is not None else t


def test_unet_step_full_width(cuda):
    """BASELINE config 3's UNet (320/640/1280, depths 0/2/10, context 77 x 2048, pooled 1280) at a 64 x 64 latent:
    the levels run at 64^2 / 32^2 / 16^2 pixels with every block of the real model."""
    import mkimage

    gh = gw = 32
    S, B = 77, 2
    u = mkimage.Unet(mkimage.UnetConfig(max_batch=B, max_gh=gh, max_gw=gw, max_context=S, slots=2))
    u.init_random(31)
    oc = OS.unet_default_cfg()
    ctxs = [rng.normal(rng.tensor_key(7, 10 + b), S * 2048).reshape(S, 2048) for b in range(B)]
    pooled = [rng.normal(rng.tensor_key(7, 20 + b), 1280) for b in range(B)]
    lats = np.stack([rng.normal(rng.tensor_key(7, 30 + b), gh * gw * 16).reshape(gh * gw, 16) * 3.0
                     for b in range(B)])
    sigmas = [1.5, 9.0]
    for b in range(B):
        u.begin(ctxs[b], pooled[b], gh, gw, slot=b)
    got = {}
    u.set_probe(lambda name, layer, a: got.__setitem__(name, a))
    eps = u.step_batch(lats, sigmas)
    u.set_probe(None)
    W = u.weights()
    u.close()
    names = ("conv_in", "in1.res", "in3.down", "in4.attn", "in5.attn", "in6.down", "in7.attn", "in8.attn",
             "mid.attn", "out0.attn", "out2.up", "out4.attn", "out5.up", "out8.res")
    for b in range(B):
        st = OS.unet_begin(oc, W, ctxs[b], pooled[b], gh, gw)
        want = {}
        ref = OS.unet_step(oc, W, st, lats[b], sigmas[b], probe=lambda n, a: want.__setitem__(n, a))
        for name in names:
            g = got[name].reshape(B, -1)[b]
            assert _cos(g, want[name]) >= 0.999, (b, name, _cos(g, want[name]))
        assert _rel(eps[b], ref) < 0.02 and _cos(eps[b], ref) >= 0.999, (b, _rel(eps[b], ref), _cos(eps[b], ref))


def test_vae_decode_full_width(cuda):
    """BASELINE config 4's decoder (128/256/512/512, two layers, the single-head d=512 mid attention) from a 32 x 32
    latent to a 256 x 256 image (mid attention over 1024 tokens)."""
    import mkimage

    gh = gw = 16
    v = mkimage.Vae(mkimage.VaeConfig(max_gh=gh, max_gw=gw))
    v.init_random(41)
    lat = rng.normal(rng.tensor_key(8, 1), gh * gw * 16).reshape(gh * gw, 16) * 0.13025
    got = {}
    v.set_probe(lambda name, layer, a: got.__setitem__(name, a))
    img = v.decode(lat, gh, gw)
    v.set_probe(None)
    W = v.weights()
    v.close()
    want = {}
    ref = OS.vae_decode(OS.vae_default_cfg(), W, lat, gh, gw, probe=lambda n, a: want.__setitem__(n, a))
    for name in ("conv_in", "mid.res0", "mid.attn", "mid.res1", "up0.res2", "up0.up", "up1.up", "up2.res0",
                 "up2.up", "up3.res2"):
        assert _cos(got[name], want[name]) >= 0.999, (name, _cos(got[name], want[name]))
    assert img.shape == (16 * gh, 16 * gw, 4) and np.all(img[..., 3] == 1.0)
    assert _rel(img, ref) < 0.01, _rel(img, ref)


def _attn_check(got, ref):
    err = np.abs(got - ref).max()
    cos = _cos(got, ref)
    assert err <= 2e-2 and cos >= 0.999, (err, cos)


@pytest.mark.parametrize("qscale", [1.0, 4.0])
def test_attention_hd128_config2_length(cuda, qscale):
    """Joint attention over L = 256 + 4096 (the 1024^2 step), text rows routed to out0; qscale 4 makes the softmax
    peaked (a few keys dominate) instead of nearly uniform."""
    import torch
    import mkimage

    B, H, S, N, hd = 1, 3, 256, 4096, 128
    L = S + N
    q = _randn((B, H, L, hd), 101, qscale, cuda, torch.bfloat16)
    k = _randn((B, H, L, hd), 102, 1.0, cuda, torch.bfloat16)
    v = _randn((B, H, L, hd), 103, 1.0, cuda, torch.bfloat16)
    out0 = torch.zeros(B * S, H * hd, dtype=torch.bfloat16, device=cuda)
    out1 = torch.zeros(B * N, H * hd, dtype=torch.bfloat16, device=cuda)
    mkimage.ops.attention(q, k, v, out0, out1, split=S)
    assert mkimage.ops.check_kernels() == 0
    ref = O.attention(_np(q)[0], _np(k)[0], _np(v)[0]).transpose(1, 0, 2).reshape(L, H * hd)
    _attn_check(_np(out0), ref[:S])
    _attn_check(_np(out1), ref[S:])


def test_attention_hd128_config5_length(cuda):
    """One head over L = 1024 + 16384 (the 2048^2 step); the oracle checks three 256-row query blocks (first, middle,
    last, the last one ragged against the 128-row tiles' ends) against all 17408 keys."""
    import torch
    import mkimage

    B, H, S, N, hd = 1, 1, 1024, 16384, 128
    L = S + N
    q = _randn((B, H, L, hd), 111, 3.0, cuda, torch.bfloat16)
    k = _randn((B, H, L, hd), 112, 1.0, cuda, torch.bfloat16)
    v = _randn((B, H, L, hd), 113, 1.0, cuda, torch.bfloat16)
    out0 = torch.zeros(B * S, H * hd, dtype=torch.bfloat16, device=cuda)
    out1 = torch.zeros(B * N, H * hd, dtype=torch.bfloat16, device=cuda)
    mkimage.ops.attention(q, k, v, out0, out1, split=S)
    assert mkimage.ops.check_kernels() == 0
    full = np.concatenate([_np(out0), _np(out1)])
    qn, kn, vn = _np(q)[0], _np(k)[0], _np(v)[0]
    for r0 in (0, L // 2 - 96, L - 256):
        ref = O.attention(qn[:, r0:r0 + 256], kn, vn)[0]
        _attn_check(full[r0:r0 + 256], ref)


def test_attention_hd64_20_heads_1024_keys(cuda):
    """The UNet's 1280-channel level at 1024^2: 20 heads of 64 over 32^2 = 1024 tokens (self) and the 77-token
    context (cross), CFG batch 2."""
    import torch
    import mkimage

    B, H, L, hd, S = 2, 20, 1024, 64, 77
    q = _randn((B, H, L, hd), 121, 2.0, cuda, torch.bfloat16)
    k = _randn((B, H, L, hd), 122, 1.0, cuda, torch.bfloat16)
    v = _randn((B, H, L, hd), 123, 1.0, cuda, torch.bfloat16)
    out = torch.zeros(B * L, H * hd, dtype=torch.bfloat16, device=cuda)
    mkimage.ops.attention(q, k, v, None, out, split=0)
    kc = _randn((B, H, S, hd), 124, 1.0, cuda, torch.bfloat16)
    vc = _randn((B, H, S, hd), 125, 1.0, cuda, torch.bfloat16)
    outc = torch.zeros(B * L, H * hd, dtype=torch.bfloat16, device=cuda)
    mkimage.ops.attention(q, kc, vc, None, outc, split=0)
    assert mkimage.ops.check_kernels() == 0
    qn, kn, vn, kcn, vcn = (_np(t) for t in (q, k, v, kc, vc))
    for b in range(B):
        ref = O.attention(qn[b], kn[b], vn[b]).transpose(1, 0, 2).reshape(L, H * hd)
        _attn_check(_np(out)[b * L:(b + 1) * L], ref)
        refc = O.attention(qn[b], kcn[b], vcn[b]).transpose(1, 0, 2).reshape(L, H * hd)
        _attn_check(_np(outc)[b * L:(b + 1) * L], refc)


@pytest.mark.parametrize("N,K", [(1280, 1280), (3840, 1280), (1280, 5120)])
def test_proj_unet_level2_1024(cuda, N, K):
    """The 32^2-level linears at 1024^2 with CFG 2 (M = 2048 rows): proj_in / out and the attention outputs,
    the fused q/k/v rows, and ff2 (K = 4 c), through the add epilogue with a residual."""
    import torch
    import mkimage

    M = 2048
    x = _randn((M, K), 131, 1.0, cuda, torch.bfloat16)
    w = _randn((N, K), 132, 0.02, cuda, torch.bfloat16)
    b = _randn((N,), 133, 0.02, cuda)
    r = _randn((M, N), 134, 1.0, cuda)
    y = mkimage.ops.proj_add(x, w, bias=b, resid=r)
    assert mkimage.ops.check_kernels() == 0
    ref = O.linear(_np(x), _np(w), _np(b)) + _np(r)
    assert np.abs(_np(y) - ref).max() <= 1e-3 * np.abs(ref).max()


def test_geglu_unet_level2_1024(cuda):
    """ff1 of the 1280-channel level (N = 8 c = 10240 interleaved hidden | gate rows) with the erf GEGLU epilogue."""
    import torch
    import mkimage

    M, c = 2048, 1280
    blk = mkimage.ops.swiglu_interleave_block()
    x = _randn((M, c), 141, 1.0, cuda, torch.bfloat16)
    wh = _randn((4 * c, c), 142, 0.03, None, torch.bfloat16)
    wg = _randn((4 * c, c), 143, 0.03, None, torch.bfloat16)
    bh = _randn((4 * c,), 144, 0.02)
    bg = _randn((4 * c,), 145, 0.02)
    wi = torch.cat([torch.cat([wh[i:i + blk], wg[i:i + blk]]) for i in range(0, 4 * c, blk)]).to(cuda)
    bi = torch.cat([torch.cat([bh[i:i + blk], bg[i:i + blk]]) for i in range(0, 4 * c, blk)]).to(cuda)
    y = mkimage.ops.proj_geglu(x, wi, bi)
    assert mkimage.ops.check_kernels() == 0
    hn = O.linear(_np(x), _np(wh), _np(bh))
    gn = O.linear(_np(x), _np(wg), _np(bg))
    ref = hn * O.gelu_erf(gn)
    assert np.abs(_np(y) - ref).max() <= 1e-2 * np.abs(ref).max()


@pytest.mark.parametrize("C,Cout,stride", [(1280, 1280, 1), (2560, 1280, 1), (640, 640, 2)])
def test_conv_unet_level2_1024(cuda, C, Cout, stride):
    """The 1280-channel level's 3x3 convolutions at 1024^2 with CFG 2: 32^2 pixels per image, the up path's
    skip-concatenated input (2560 channels), and the stride-2 downsample from 64^2."""
    import torch
    import mkimage

    B, H = 2, 32 * stride
    x = _randn((B, H, H, C), 151, 1.0, cuda, torch.bfloat16)
    w = _randn((Cout, 9 * C), 152, 0.01, cuda, torch.bfloat16)
    bias = _randn((Cout,), 153, 0.1, cuda)
    Ho = (H - 1) // stride + 1
    resid = _randn((B, Ho, Ho, Cout), 154, 1.0, cuda)
    y = mkimage.ops.conv2d(x, w, taps=9, stride=stride, bias=bias, resid=resid)
    assert mkimage.ops.check_kernels() == 0
    ref = O.conv2d_nhwc(_np(x), _np(w).reshape(Cout, 9, C), stride, 9, _np(bias)) + _np(resid)
    assert np.abs(_np(y) - ref).max() <= 1e-3 * np.abs(ref).max()
