"""Parity of the SDXL-path kernels: implicit-GEMM convolution (3x3 stride 1 / 2, 1x1; narrow and ragged images),
GroupNorm(+SiLU), the add / head-scatter / GEGLU projection epilogues, and head-dim-64 attention (self and 77-key
cross), each against the numpy oracle on identical inputs.

Tolerances: fp32-output kernels accumulate in fp32 like the oracle (max-abs <= 1e-3 of the output scale); bf16
outputs <= 1e-2 of the scale; attention <= 2e-2 with cosine >= 0.999."""

import numpy as np
import pytest

from oracle import ops as O

pytestmark = pytest.mark.gpu


def _t(shape, seed, scale=1.0, dev=None):
    import torch

    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(dev)


def _np(t):
    return t.float().cpu().numpy()


@pytest.mark.parametrize("B,H,W,C,Cout,taps,stride", [
    (2, 16, 32, 64, 96, 9, 1),     # 3x3, tiles 8 x 16
    (1, 32, 32, 128, 64, 9, 2),    # stride 2 (downsample)
    (1, 12, 8, 64, 64, 9, 1),      # width 8 (tiles 16 x 8), ragged rows
    (1, 16, 16, 128, 256, 1, 1),   # 1x1 (one CTA-pair tile)
    (2, 64, 64, 320, 320, 9, 1),   # SDXL level-0 width (CTA pairs, 160-wide tiles)
    (1, 17, 32, 64, 32, 9, 2),     # odd input height, stride 2
    (1, 24, 16, 64, 256, 9, 1),    # CTA pairs over an odd count (3) of 128-pixel tiles
])
def test_conv2d(cuda, B, H, W, C, Cout, taps, stride):
    import torch
    import mkimage

    x = _t((B, H, W, C), 1, dev=cuda).to(torch.bfloat16)
    w = _t((Cout, taps * C), 2, 0.05, cuda).to(torch.bfloat16)
    bias = _t((Cout,), 3, 0.1, cuda)
    Ho = (H - 1) // stride + 1 if taps == 9 else H
    Wo = (W - 1) // stride + 1 if taps == 9 else W
    addvec = _t((B, Cout), 4, 0.1, cuda)
    resid = _t((B, Ho, Wo, Cout), 5, 1.0, cuda)
    y = mkimage.ops.conv2d(x, w, taps=taps, stride=stride, bias=bias, addvec=addvec, resid=resid)
    assert mkimage.ops.check_kernels() == 0
    ref = O.conv2d_nhwc(_np(x), _np(w).reshape(Cout, taps, C), stride, taps, _np(bias))
    ref = ref + _np(addvec)[:, None, None, :] + _np(resid)
    assert y.shape == (B, Ho, Wo, Cout)
    err = np.abs(_np(y) - ref).max() / np.abs(ref).max()
    assert err < 1e-3, err
    yb = mkimage.ops.conv2d(x, w, taps=taps, stride=stride, out_f32=False)
    refb = O.conv2d_nhwc(_np(x), _np(w).reshape(Cout, taps, C), stride, taps)
    assert np.abs(_np(yb) - refb).max() < 1e-2 * np.abs(refb).max()


@pytest.mark.parametrize("B,HW,C,silu,eps", [(2, 300, 320, True, 1e-5), (1, 4096, 640, False, 1e-6),
                                              (2, 64, 2560, True, 1e-5), (1, 1000, 128, True, 1e-6)])
def test_group_norm(cuda, B, HW, C, silu, eps):
    import mkimage

    x = (_t((B, HW, C), 6, 2.0, cuda) + 3.0)  # a non-zero mean checks the variance's numerics
    g = 1 + _t((C,), 7, 0.1, cuda)
    b = _t((C,), 8, 0.1, cuda)
    y = mkimage.ops.group_norm(x, g, b, 32, eps, silu)
    assert mkimage.ops.check_kernels() == 0
    ref = O.group_norm_nhwc(_np(x), _np(g), _np(b), 32, eps, silu)
    assert np.abs(_np(y) - ref).max() < 2e-2 * max(1.0, np.abs(ref).max())


def test_proj_add_in_place(cuda):
    import torch
    import mkimage

    M, N, K = 700, 640, 320
    x = _t((M, K), 9, 1.0, cuda).to(torch.bfloat16)
    w = _t((N, K), 10, 0.05, cuda).to(torch.bfloat16)
    b = _t((N,), 11, 0.1, cuda)
    r0 = _t((M, N), 12, 1.0, cuda)
    r = r0.clone()
    mkimage.ops.proj_add(x, w, b, resid=r, out=r)
    ref = O.linear(_np(x), _np(w), _np(b)) + _np(r0)
    assert np.abs(_np(r) - ref).max() < 1e-3 * np.abs(ref).max()


def test_proj_heads_hd64(cuda):
    import torch
    import mkimage

    B, N_tok, heads, hd, K = 2, 200, 5, 64, 320
    D = heads * hd
    x = _t((B * N_tok, K), 13, 1.0, cuda).to(torch.bfloat16)
    w = _t((3 * D, K), 14, 0.05, cuda).to(torch.bfloat16)
    qh = torch.zeros(B, heads, N_tok, hd, dtype=torch.bfloat16, device=cuda)
    kh, vh = torch.zeros_like(qh), torch.zeros_like(qh)
    mkimage.ops.proj_heads(x, w, None, qh, kh, vh, 0, D, N_tok, 0)
    y = O.linear(_np(x), _np(w)).reshape(B, N_tok, 3, heads, hd)
    for i, t in enumerate((qh, kh, vh)):
        ref = y[:, :, i].transpose(0, 2, 1, 3)
        assert np.abs(_np(t) - ref).max() < 1e-2 * np.abs(ref).max()
    # k and v only (part0 = 1), e.g. the cached cross-attention context
    kc, vc = torch.zeros(B, heads, 77, hd, dtype=torch.bfloat16, device=cuda), torch.zeros(B, heads, 77, hd, dtype=torch.bfloat16, device=cuda)
    ctx = _t((B * 77, K), 15, 1.0, cuda).to(torch.bfloat16)
    wkv = _t((2 * D, K), 16, 0.05, cuda).to(torch.bfloat16)
    mkimage.ops.proj_heads(ctx, wkv, None, None, kc, vc, 1, D, 77, 0)
    y = O.linear(_np(ctx), _np(wkv)).reshape(B, 77, 2, heads, hd)
    assert np.abs(_np(kc) - y[:, :, 0].transpose(0, 2, 1, 3)).max() < 1e-2 * np.abs(y).max()
    assert np.abs(_np(vc) - y[:, :, 1].transpose(0, 2, 1, 3)).max() < 1e-2 * np.abs(y).max()


def test_proj_geglu(cuda):
    import torch
    import mkimage

    M, F, K = 300, 512, 320
    B = mkimage.ops.swiglu_interleave_block()
    x = _t((M, K), 17, 1.0, cuda).to(torch.bfloat16)
    wh = _t((F, K), 18, 0.05).to(torch.bfloat16)
    wg = _t((F, K), 19, 0.05).to(torch.bfloat16)
    bh, bg = _t((F,), 20, 0.1), _t((F,), 21, 0.1)
    wi = torch.cat([torch.cat([wh[j:j + B], wg[j:j + B]]) for j in range(0, F, B)]).to(cuda)
    bi = torch.cat([torch.cat([bh[j:j + B], bg[j:j + B]]) for j in range(0, F, B)]).to(cuda)
    y = mkimage.ops.proj_geglu(x, wi, bi)
    ref = O.linear(_np(x), _np(wh), _np(bh)) * O.gelu_erf(O.linear(_np(x), _np(wg), _np(bg)))
    assert np.abs(_np(y) - ref).max() < 1e-2 * np.abs(ref).max()


@pytest.mark.parametrize("B,H,Lq,Lk", [(2, 10, 4096, 4096), (2, 20, 1024, 77), (1, 5, 300, 300)])
def test_attention_hd64(cuda, B, H, Lq, Lk):
    import torch
    import mkimage

    q = _t((B, H, Lq, 64), 22, 1.0, cuda).to(torch.bfloat16)
    k = _t((B, H, Lk, 64), 23, 1.0, cuda).to(torch.bfloat16)
    v = _t((B, H, Lk, 64), 24, 1.0, cuda).to(torch.bfloat16)
    out = torch.zeros(B * Lq, H * 64, dtype=torch.bfloat16, device=cuda)
    mkimage.ops.attention(q, k, v, None, out, split=0)
    assert mkimage.ops.check_kernels() == 0
    qn, kn, vn = _np(q), _np(k), _np(v)
    for b in range(B):
        ref = O.attention(qn[b], kn[b], vn[b]).transpose(1, 0, 2).reshape(Lq, H * 64)
        got = _np(out[b * Lq:(b + 1) * Lq])
        assert np.abs(got - ref).max() < 2e-2
        assert (got * ref).sum() / np.sqrt((got ** 2).sum() * (ref ** 2).sum()) > 0.999
