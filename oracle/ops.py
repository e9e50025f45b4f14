"""Row and matrix operations of the reference's denoiser, restated in numpy (fp32 unless noted).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py). Each function cites the reference call site it follows."""

import numpy as np


def bf16_round(a):
    """Round fp32 values to the nearest bf16 (ties to even), returned as fp32."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32).reshape(a.shape)


def linear(x, w, b=None):
    """y = x w^T + b: the runtime's proj() with W stored [out][in] (qwen_image.cpp:99-105 stacks rows that way)."""
    y = np.asarray(x, np.float32) @ np.asarray(w, np.float32).T
    if b is not None:
        y = y + np.asarray(b, np.float32)
    return y.astype(np.float32)


def gelu_tanh(x):
    """GELU, tanh approximation (the `gelu_tanh` kernel applied at qwen_image.cpp:211)."""
    x = np.asarray(x, np.float32)
    return (0.5 * x * (1.0 + np.tanh(0.7978845608028654 * (x + 0.044715 * x * x * x)))).astype(np.float32)


def silu(x):
    """x * sigmoid(x) (the `silu` kernel, qwen_image.cpp:198,202)."""
    x = np.asarray(x, np.float32)
    return (x / (1.0 + np.exp(-x))).astype(np.float32)


def rms_norm(x, w, eps=1e-6):
    """x / rms(x) * w over the last axis (runtime norm(), qwen_image.cpp:208; per-head norms :226-242)."""
    x = np.asarray(x, np.float32)
    ms = np.mean(x.astype(np.float64) ** 2, axis=-1, keepdims=True)
    return (x / np.sqrt(ms + eps).astype(np.float32) * np.asarray(w, np.float32)).astype(np.float32)


def ln_modulate(x, scale, shift=None, eps=1e-6):
    """LayerNorm without affine, times (1 + scale), plus shift (`ln_modulate`, src/kernels/image.metal:33-53; the
    reference has no shift, Qwen-Image-1's AdaLN adds one)."""
    x = np.asarray(x, np.float32)
    x64 = x.astype(np.float64)
    mean = x64.mean(axis=-1, keepdims=True)
    var = ((x64 - mean) ** 2).mean(axis=-1, keepdims=True)
    y = ((x64 - mean) / np.sqrt(var + eps)).astype(np.float32) * (1.0 + np.asarray(scale, np.float32))
    if shift is not None:
        y = y + np.asarray(shift, np.float32)
    return y.astype(np.float32)


def rope_pairs(x, cs):
    """Rotate interleaved pairs (x[2i], x[2i+1]) by the table cs[..., i, (cos, sin)] (RoPE mode 2 of
    heads_norm_half, qwen_image.cpp:226-242; table built by rope3, :31-45). x [..., L, 128], cs [L, 64, 2]."""
    x = np.asarray(x, np.float32)
    x0, x1 = x[..., 0::2], x[..., 1::2]
    c, s = cs[..., 0], cs[..., 1]
    out = np.empty_like(x)
    out[..., 0::2] = x0 * c - x1 * s
    out[..., 1::2] = x0 * s + x1 * c
    return out


def attention(q, k, v, mask=None):
    """softmax(q k^T / sqrt(d)) v per head (runtime attention(), qwen_image.cpp:271). q [H][Lq][d], k/v [H][Lk][d];
    mask [Lq][Lk] boolean (True = may attend) or None."""
    q = np.asarray(q, np.float32)
    d = q.shape[-1]
    out = np.empty(q.shape, np.float32)
    for h in range(q.shape[0]):
        s = (q[h] @ np.asarray(k[h], np.float32).T) * np.float32(1.0 / np.sqrt(d))
        if mask is not None:
            s = np.where(mask, s, -np.inf)
        s = s - s.max(axis=-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=-1, keepdims=True)
        out[h] = p @ np.asarray(v[h], np.float32)
    return out


def timestep_sinusoid(sigma, dim=256):
    """Cos-first sinusoid of 1000 * sigma (qwen_image.cpp:179-187): freq_i = exp(-ln(10000) i / (dim/2))."""
    half = dim // 2
    i = np.arange(half, dtype=np.float32)
    freq = np.exp(-np.log(np.float32(10000.0)) * i / np.float32(half)).astype(np.float32)
    arg = np.float32(1000.0 * sigma) * freq
    return np.concatenate([np.cos(arg), np.sin(arg)]).astype(np.float32)


def gelu_erf(x):
    """GELU with the exact erf (SDXL's GEGLU, src/kernels/image.metal:451-463,476-484; the oracle uses the exact erf
    rather than the reference's fitted one)."""
    from math import erf

    x = np.asarray(x, np.float64)
    v = np.vectorize(erf)(x * 0.7071067811865476) if x.size < 4096 else _erf_np(x * 0.7071067811865476)
    return (0.5 * x * (1.0 + v)).astype(np.float32)


def _erf_np(z):
    import scipy.special

    return scipy.special.erf(z)


def conv2d_nhwc(x, w, stride=1, taps=9, bias=None):
    """Convolution of channels-last x [B][H][W][C] with w [Cout][taps][C] (taps 9: 3x3, padding 1; taps 1: 1x1):
    the runtime's conv (im2col + GEMM, docs/architecture.md:178; called at sdxl.cpp:729-735), in fp32."""
    x = np.asarray(x, np.float32)
    B, H, W, C = x.shape
    Cout = w.shape[0]
    if taps == 1:
        y = x.reshape(-1, C) @ np.asarray(w, np.float32).reshape(Cout, C).T
        y = y.reshape(B, H, W, Cout)
    else:
        xp = np.zeros((B, H + 2, W + 2, C), np.float32)
        xp[:, 1:H + 1, 1:W + 1] = x
        Ho, Wo = (H - 1) // stride + 1, (W - 1) // stride + 1
        cols = np.empty((B, Ho, Wo, 9, C), np.float32)
        for dy in range(3):
            for dx in range(3):
                cols[:, :, :, dy * 3 + dx] = xp[:, dy:dy + stride * (Ho - 1) + 1:stride, dx:dx + stride * (Wo - 1) + 1:stride]
        y = cols.reshape(-1, 9 * C) @ np.asarray(w, np.float32).reshape(Cout, 9 * C).T
        y = y.reshape(B, Ho, Wo, Cout)
    if bias is not None:
        y = y + np.asarray(bias, np.float32)
    return y.astype(np.float32)


def group_norm_nhwc(x, gamma, beta, groups=32, eps=1e-5, silu=False):
    """GroupNorm over channels-last x [B][..][C]: statistics per sample over the group's C/groups consecutive
    channels and all pixels (the runtime's group_norm, sdxl.cpp:728; optional fused SiLU, its `true` argument)."""
    x = np.asarray(x, np.float32)
    B, C = x.shape[0], x.shape[-1]
    xr = x.reshape(B, -1, groups, C // groups).astype(np.float64)
    mean = xr.mean(axis=(1, 3), keepdims=True)
    var = ((xr - mean) ** 2).mean(axis=(1, 3), keepdims=True)
    y = ((xr - mean) / np.sqrt(var + eps)).reshape(x.shape) * np.asarray(gamma, np.float64)
    if beta is not None:
        y = y + np.asarray(beta, np.float64)
    y = y.astype(np.float32)
    return silu_(y) if silu else y


def silu_(x):
    return (x / (1.0 + np.exp(-x.astype(np.float64)))).astype(np.float32)


def upsample2x_nhwc(x):
    """Nearest 2x (upsample2x, src/kernels/image.metal:77-84)."""
    return np.repeat(np.repeat(np.asarray(x, np.float32), 2, axis=1), 2, axis=2)


def lora_merge(W, A, B, scale, alpha=None):
    """A LoRA pair merged into a bf16 matrix: W + scale * (alpha / rank) * B A, rounded to bf16 (alpha None: 1).

    The reference adds adapters by module (Engine::add_lora, src/image/engine.hpp:195-197), each module a row range
    of a stacked matrix (QwenImage::lora_target, src/image/qwen_image.cpp:295-331); the merge itself runs in the
    absent mako-common runtime, so this restates the standard LoRA update (Hu et al., 2021) on those rows."""
    W = np.asarray(W, np.float32)
    A = np.asarray(A, np.float64)
    B = np.asarray(B, np.float64)
    s = scale * (alpha / A.shape[0] if alpha is not None else 1.0)
    return bf16_round((W.astype(np.float64) + s * (B @ A)).astype(np.float32))
