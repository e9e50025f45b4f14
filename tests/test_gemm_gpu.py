"""Parity of the tcgen05 projection kernels (mkb_proj*) against the numpy oracle on identical bf16 inputs.

Tolerance: the kernels accumulate in fp32 like the oracle; the only differences are summation order and the final
bf16 rounding of bf16 outputs, so max-abs error <= 1e-2 relative to the output scale (fp32 outputs: 1e-4)."""

import numpy as np
import pytest

from oracle import ops as O

pytestmark = pytest.mark.gpu


def _bf16(t):
    return t.to(__import__("torch").bfloat16)


def _np(t):
    return t.float().cpu().numpy()


def _rand(shape, seed, scale=1.0):
    import torch

    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g) * scale


# Tile widths the makespan chooser picks for these shapes: 64, 64, 64, 128, 256 on CTA pairs, 160, 192.
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 512, 320), (1, 3072, 256), (1000, 1536, 3072),
                                   (4352, 3072, 3072), (2048, 1280, 320), (2304, 1536, 192)])
@pytest.mark.parametrize("out_f32", [False, True])
def test_proj(cuda, M, N, K, out_f32):
    import mkimage

    x = _bf16(_rand((M, K), 1)).to(cuda)
    w = _bf16(_rand((N, K), 2, 0.02)).to(cuda)
    b = _rand((N,), 3, 0.02).to(cuda)
    y = mkimage.ops.proj(x, w, b, out_f32=out_f32)
    assert mkimage.ops.check_kernels() == 0
    ref = O.linear(_np(x), _np(w), _np(b))
    got = _np(y)
    scale = np.abs(ref).max()
    err = np.abs(got - ref).max() / scale
    assert err < (1e-4 if out_f32 else 1e-2), err


@pytest.mark.parametrize("act", [1, 2])
def test_proj_act(cuda, act):
    import mkimage

    M, N, K = 256, 1024, 512
    x = _bf16(_rand((M, K), 4)).to(cuda)
    w = _bf16(_rand((N, K), 5, 0.05)).to(cuda)
    b = _rand((N,), 6, 0.1).to(cuda)
    y = mkimage.ops.proj(x, w, b, act=act, out_f32=True)
    lin = O.linear(_np(x), _np(w), _np(b))
    ref = O.gelu_tanh(lin) if act == 1 else O.silu(lin)
    # tanh runs on the SFU (tanh.approx, relative error ~2^-11), well below the bf16 rounding the model applies
    assert np.abs(_np(y) - ref).max() < 1e-3 * max(1.0, np.abs(ref).max())


@pytest.mark.parametrize("tanh_gate", [False, True])
def test_proj_gate_add(cuda, tanh_gate):
    import mkimage

    M, N, K, rps = 640, 768, 384, 320  # two samples of 320 rows
    x = _bf16(_rand((M, K), 7)).to(cuda)
    w = _bf16(_rand((N, K), 8, 0.05)).to(cuda)
    b = _rand((N,), 9, 0.1).to(cuda)
    gate = _rand((2, N), 10, 0.5).to(cuda)
    r0 = _rand((M, N), 11).to(cuda)
    r = r0.clone()
    mkimage.ops.proj_gate_add(x, w, r, gate, b, rows_per_sample=rps, tanh_gate=tanh_gate)
    y = O.linear(_np(x), _np(w), _np(b))
    g = _np(gate)
    g = np.tanh(g) if tanh_gate else g
    ref = _np(r0) + np.repeat(g, rps, axis=0) * y
    assert np.abs(_np(r) - ref).max() < 1e-4 * np.abs(ref).max()


def test_proj_qkv_heads(cuda):
    import torch
    import mkimage

    heads, S, N_img, samples = 4, 40, 96, 2
    D = heads * 128
    L = S + N_img
    K = 256
    x = _bf16(_rand((samples * N_img, K), 12)).to(cuda)  # the image stream of two samples
    w = _bf16(_rand((3 * D, K), 13, 0.05)).to(cuda)
    b = _rand((3 * D,), 14, 0.1).to(cuda)
    nq = (1 + _rand((128,), 15, 0.1)).to(cuda)
    nk = (1 + _rand((128,), 16, 0.1)).to(cuda)
    ang = _rand((L, 64), 17, 3.0)
    rope = torch.stack([ang.cos(), ang.sin()], -1).contiguous().to(cuda)
    qh = torch.zeros(samples, heads, L, 128, dtype=torch.bfloat16, device=cuda)
    kh, vh = torch.zeros_like(qh), torch.zeros_like(qh)
    mkimage.ops.proj_qkv_heads(x, w, b, nq, nk, rope, qh, kh, vh, rows_per_sample=N_img, pos_offset=S)
    assert mkimage.ops.check_kernels() == 0
    y = O.linear(_np(x), _np(w), _np(b)).reshape(samples, N_img, 3, heads, 128)
    cs = _np(rope)[S:]
    for which, (out, wn) in enumerate([(qh, nq), (kh, nk), (vh, None)]):
        ref = y[:, :, which].transpose(0, 2, 1, 3)  # [samples][heads][N_img][128]
        if wn is not None:
            ref = O.rope_pairs(O.rms_norm(ref, _np(wn)), cs)
        got = _np(out)[:, :, S:]
        assert np.abs(got - ref).max() < 2e-2 * max(1.0, np.abs(ref).max()), which
        assert np.abs(_np(out)[:, :, :S]).max() == 0  # text rows untouched


def test_proj_swiglu(cuda):
    import torch
    import mkimage

    M, F, K = 384, 512, 256
    B = mkimage.ops.swiglu_interleave_block()
    x = _bf16(_rand((M, K), 18)).to(cuda)
    wg = _bf16(_rand((F, K), 19, 0.05))
    wu = _bf16(_rand((F, K), 20, 0.05))
    wi = torch.cat([torch.cat([wg[j:j + B], wu[j:j + B]]) for j in range(0, F, B)]).to(cuda)
    y = mkimage.ops.proj_swiglu(x, wi)
    ref = O.silu(O.linear(_np(x), _np(wg))) * O.linear(_np(x), _np(wu))
    assert np.abs(_np(y) - ref).max() < 1e-2 * np.abs(ref).max()
