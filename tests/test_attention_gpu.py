"""Parity of the tcgen05 flash-attention kernel (mkb_attention) against the numpy oracle.

Tolerance: P is rounded to bf16 before the P.V product and outputs are bf16, so max-abs <= 2e-2 (outputs are
O(1) averages of unit-variance values) and cosine >= 0.999 per row block."""

import numpy as np
import pytest

from oracle import ops as O

pytestmark = pytest.mark.gpu


def _heads(shape, seed, cuda):
    import torch

    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).to(torch.bfloat16).to(cuda)


def _run(cuda, B, H, S, N, mask, later=False):
    import torch
    import mkimage

    L = S + N
    q = _heads((B, H, L, 128), 1, cuda)
    k = _heads((B, H, L, 128), 2, cuda)
    v = _heads((B, H, L, 128), 3, cuda)
    out0 = torch.zeros(B * S, H * 128, dtype=torch.bfloat16, device=cuda)
    out1 = torch.zeros(B * N, H * 128, dtype=torch.bfloat16, device=cuda)
    if later:  # queries: the image rows only, at joint positions S..L-1
        qi = q[:, :, S:].contiguous()
        mkimage.ops.attention(qi, k, v, None, out1, split=S, q_pos0=S, mask=mask, cond_len=S)
    else:
        mkimage.ops.attention(q, k, v, out0, out1, split=S, mask=mask, cond_len=S)
    assert mkimage.ops.check_kernels() == 0
    qn, kn, vn = (t.float().cpu().numpy() for t in (q, k, v))
    pos = np.arange(L)
    m = None
    if mask == mkimage.ops.MASK_COND_CAUSAL:
        m = (pos[:, None] >= S) | (pos[None, :] <= pos[:, None])  # text rows causal, image rows see all
    for b in range(B):
        ref = O.attention(qn[b], kn[b], vn[b], m)  # [H][L][128]
        ref = ref.transpose(1, 0, 2).reshape(L, H * 128)
        got_img = out1[b * N:(b + 1) * N].float().cpu().numpy()
        err = np.abs(got_img - ref[S:]).max()
        assert err < 2e-2, err
        cos = (got_img * ref[S:]).sum() / np.sqrt((got_img ** 2).sum() * (ref[S:] ** 2).sum())
        assert cos > 0.999
        if not later:
            got_txt = out0[b * S:(b + 1) * S].float().cpu().numpy()
            assert np.abs(got_txt - ref[:S]).max() < 2e-2


@pytest.mark.parametrize("B,H,S,N", [(1, 1, 128, 128), (2, 3, 44, 256), (1, 2, 77, 1000)])
def test_attention_joint(cuda, B, H, S, N):
    _run(cuda, B, H, S, N, 0)


@pytest.mark.parametrize("B,H,S,N", [(2, 3, 44, 256), (1, 2, 200, 300)])
def test_attention_cond_causal(cuda, B, H, S, N):
    _run(cuda, B, H, S, N, 1)


def test_attention_cond_causal_cached_text(cuda):
    _run(cuda, 2, 2, 130, 260, 1, later=True)


def test_attention_rejects_bad_routing(cuda):
    import torch
    import mkimage

    q = torch.zeros(1, 1, 256, 128, dtype=torch.bfloat16, device=cuda)
    out1 = torch.zeros(100, 128, dtype=torch.bfloat16, device=cuda)  # too few rows for 256 queries
    with pytest.raises(mkimage.MkbError):
        mkimage.ops.attention(q, q, q, None, out1, split=0)


@pytest.mark.parametrize("hd,G,B,H,S,N", [(128, 2, 2, 3, 100, 412), (128, 4, 1, 2, 64, 960), (64, 2, 2, 2, 77, 435)])
def test_attention_kv_shards_bit_exact(cuda, hd, G, B, H, S, N):
    """K/V split into G shards of L/G rows (K and V of a shard interleaved, as the sequence-parallel step gathers
    them) gives bit-identical outputs to the unsplit call: same key tiles, same order."""
    import torch
    import mkimage

    L = S + N
    Lg = L // G
    assert L % G == 0 and Lg % 128 == 0
    q = _heads((B, H, L, hd), 11, cuda)
    k = _heads((B, H, L, hd), 12, cuda)
    v = _heads((B, H, L, hd), 13, cuda)
    ref0 = torch.zeros(B * S, H * hd, dtype=torch.bfloat16, device=cuda)
    ref1 = torch.zeros(B * N, H * hd, dtype=torch.bfloat16, device=cuda)
    mkimage.ops.attention(q, k, v, ref0, ref1, split=S)
    # [G][2][B*H][Lg][hd]: shard g holds key rows [g*Lg, (g+1)*Lg) of every head, K then V.
    kv = torch.empty(G, 2, B * H, Lg, hd, dtype=torch.bfloat16, device=cuda)
    for g in range(G):
        kv[g, 0] = k.reshape(B * H, L, hd)[:, g * Lg:(g + 1) * Lg]
        kv[g, 1] = v.reshape(B * H, L, hd)[:, g * Lg:(g + 1) * Lg]
    out0 = torch.zeros_like(ref0)
    out1 = torch.zeros_like(ref1)
    mkimage.ops.attention_kv_shards(q, kv[0, 0], kv[0, 1], out0, out1, split=S, Lk=L, kv_shard_rows=Lg,
                                    kv_plane_stride=2 * B * H)
    assert mkimage.ops.check_kernels() == 0
    assert torch.equal(out0, ref0) and torch.equal(out1, ref1)
    # The queries of one shard alone (a sequence-parallel rank's rows), routed past the text rows.
    r = G - 1
    qr = q[:, :, r * Lg:(r + 1) * Lg].contiguous()
    outr = torch.zeros(B * Lg, H * hd, dtype=torch.bfloat16, device=cuda)
    mkimage.ops.attention_kv_shards(qr, kv[0, 0], kv[0, 1], None, outr, split=r * Lg, Lk=L, kv_shard_rows=Lg,
                                    kv_plane_stride=2 * B * H, q_pos0=r * Lg)
    assert mkimage.ops.check_kernels() == 0
    for b in range(B):
        assert torch.equal(outr[b * Lg:(b + 1) * Lg], ref1[b * N + r * Lg - S:b * N + (r + 1) * Lg - S])


@pytest.mark.parametrize("hd,G,B,H,S,N", [(128, 2, 2, 3, 100, 412), (128, 4, 1, 2, 64, 960)])
def test_attention_kv_arriving(cuda, hd, G, B, H, S, N):
    """Shards that other ranks copy in during the launch (mkb_attention_kv_arriving): with every ready flag at the
    expected value, each shard's queries (a rank's rows, own_shard = that rank) read the keys starting at their own
    shard and wrapping round. Only the online softmax's rounding differs from the in-order call: outputs within the
    oracle tolerance of it (max-abs 2e-2, cosine 0.9999), and against the oracle itself."""
    import torch
    import mkimage

    L = S + N
    Lg = L // G
    q = _heads((B, H, L, hd), 21, cuda)
    k = _heads((B, H, L, hd), 22, cuda)
    v = _heads((B, H, L, hd), 23, cuda)
    kv = torch.empty(G, 2, B * H, Lg, hd, dtype=torch.bfloat16, device=cuda)
    for g in range(G):
        kv[g, 0] = k.reshape(B * H, L, hd)[:, g * Lg:(g + 1) * Lg]
        kv[g, 1] = v.reshape(B * H, L, hd)[:, g * Lg:(g + 1) * Lg]
    ready = torch.full((G,), 7, dtype=torch.int64, device=cuda)
    expect = torch.tensor([7], dtype=torch.int64, device=cuda)
    qn, kn, vn = (t.float().cpu().numpy() for t in (q, k, v))
    for r in range(G):
        qr = q[:, :, r * Lg:(r + 1) * Lg].contiguous()
        want = torch.zeros(B * Lg, H * hd, dtype=torch.bfloat16, device=cuda)
        got = torch.zeros_like(want)
        mkimage.ops.attention_kv_shards(qr, kv[0, 0], kv[0, 1], None, want, split=r * Lg, Lk=L, kv_shard_rows=Lg,
                                        kv_plane_stride=2 * B * H, q_pos0=r * Lg)
        mkimage.ops.attention_kv_arriving(qr, kv[0, 0], kv[0, 1], None, got, split=r * Lg, Lk=L,
                                          kv_shard_rows=Lg, kv_plane_stride=2 * B * H, own_shard=r,
                                          shard_ready=ready, shard_expect=expect, q_pos0=r * Lg)
        assert mkimage.ops.check_kernels() == 0
        a, w = got.float().cpu().numpy(), want.float().cpu().numpy()
        assert np.abs(a - w).max() < 2e-2
        assert (a * w).sum() / np.sqrt((a * a).sum() * (w * w).sum()) > 0.9999
        for b in range(B):
            ref = O.attention(qn[b, :, r * Lg:(r + 1) * Lg], kn[b], vn[b], None)
            ref = ref.transpose(1, 0, 2).reshape(Lg, H * hd)
            assert np.abs(a[b * Lg:(b + 1) * Lg] - ref).max() < 2e-2


def test_attention_kv_arriving_flag_never_set(cuda):
    """A shard whose ready flag nobody raises: every CTA gives up after the bounded wait (2 s for the first, at once
    for the others once the status bit is set), the launch reports MKB_ERR_KERNEL with the shard-wait bit (0x100),
    and the same context then runs the call correctly once the flag is raised."""
    import ctypes
    import time

    import torch
    import mkimage

    G, B, H, Lg, hd = 2, 1, 2, 256, 128
    L = G * Lg
    q = _heads((B, H, Lg, hd), 31, cuda)
    kv = _heads((G, 2, B * H, Lg, hd), 32, cuda)
    ready = torch.tensor([5, 4], dtype=torch.int64, device=cuda)  # shard 1 short of the expected 5
    expect = torch.tensor([5], dtype=torch.int64, device=cuda)
    out = torch.zeros(B * Lg, H * hd, dtype=torch.bfloat16, device=cuda)
    assert mkimage.ops.check_kernels() == 0
    t0 = time.time()
    mkimage.ops.attention_kv_arriving(q, kv[0, 0], kv[0, 1], None, out, split=0, Lk=L, kv_shard_rows=Lg,
                                      kv_plane_stride=2 * B * H, own_shard=0, shard_ready=ready, shard_expect=expect)
    bits = ctypes.c_uint32()
    code = mkimage.lib.mkb_check_kernels(ctypes.byref(bits))
    elapsed = time.time() - t0
    assert code == 4, (code, mkimage.lib.mkb_last_error())  # MKB_ERR_KERNEL
    assert bits.value & 0x100, hex(bits.value)
    assert 1.5 < elapsed < 60, elapsed
    assert mkimage.ops.check_kernels() == 0
    ready[1] = 5
    mkimage.ops.attention_kv_arriving(q, kv[0, 0], kv[0, 1], None, out, split=0, Lk=L, kv_shard_rows=Lg,
                                      kv_plane_stride=2 * B * H, own_shard=0, shard_ready=ready, shard_expect=expect)
    assert mkimage.ops.check_kernels() == 0
    want = torch.zeros_like(out)
    mkimage.ops.attention_kv_shards(q, kv[0, 0], kv[0, 1], None, want, split=0, Lk=L, kv_shard_rows=Lg,
                                    kv_plane_stride=2 * B * H)
    assert (out.float() - want.float()).abs().max().item() < 2e-2


@pytest.mark.parametrize("d,n", [(512, 300), (512, 1024), (256, 77), (256, 640)])
def test_attention_wide_single_head(cuda, d, n):
    """mkb_attention_wide (the VAE mid block's single-head attention at 256 / 512 channels) against the oracle: q, k
    and v side by side in rows of 3d, ragged n (keys past the last full tile masked), both output halves."""
    import torch
    import mkimage

    qkv = _heads((n, 3 * d), 41 + d, cuda)
    out = mkimage.ops.attention_wide(qkv, d)
    assert mkimage.ops.check_kernels() == 0
    x = qkv.float().cpu().numpy()
    q, k, v = x[:, :d], x[:, d:2 * d], x[:, 2 * d:]
    ref = O.attention(q[None], k[None], v[None], None)[0]
    got = out.float().cpu().numpy()
    err = np.abs(got - ref).max()
    cos = (got * ref).sum() / np.sqrt((got ** 2).sum() * (ref ** 2).sum())
    assert err < 2e-2 and cos > 0.999, (err, cos)


_PAIR_CHILD = r"""
import sys
sys.path[:0] = [{root!r}, {pkg!r}]
import torch
import tests.test_attention_gpu as t
cuda = torch.device("cuda", 0)
t._run(cuda, 2, 3, 44, 256, 0)
t._run(cuda, 1, 2, 77, 1000, 0)
t._run(cuda, 2, 3, 44, 256, 1)
t._run(cuda, 2, 2, 130, 260, 1, later=True)
t.test_attention_kv_shards_bit_exact(cuda, 128, 4, 1, 2, 64, 960)
t.test_attention_kv_arriving(cuda, 128, 2, 2, 3, 100, 412)
print("PAIR_OK")
"""


def test_attention_cta_pairs(cuda):
    """The CTA-pair form of the head-dim-128 kernel (MKB_ATTN_PAIR=1, read once per process, so in a child): joint,
    condition-causal and cached-text masks, key shards and arriving shards, against the oracle as above."""
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = _PAIR_CHILD.format(root=root, pkg=os.path.join(root, "mako-image_b200"))
    r = subprocess.run([sys.executable, "-c", code], env=dict(os.environ, MKB_ATTN_PAIR="1"), capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0 and "PAIR_OK" in r.stdout, (r.stdout[-2000:], r.stderr[-4000:])
