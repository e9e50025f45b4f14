"""Host logic of the sequence-parallel step, on the CPU.

mkb_dit_sp_rows is the partition the library uses: the shards must tile every sample's joint rows exactly, with all
text rows on rank 0. The velocity exchange (each rank places its image rows at their shard positions, an
all-gather, then every shard's image rows back in token order) is replayed here with a world-size-2 gloo group over
the same partition, so the index arithmetic is checked with a real collective; so is the head-parallel exchange's
layout (the spans the QKV epilogue fills, the shard planes the attention reads, the output spans and columns), with
two and four gloo ranks."""

import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "mako-image_b200"))


@pytest.mark.parametrize("S,N,world", [(1024, 16384, 1), (1024, 16384, 2), (1024, 16384, 4), (1024, 16384, 8),
                                       (256, 4096, 2), (128, 384, 2)])
def test_partition_tiles_joint_rows(S, N, world):
    import mkimage

    L = S + N
    seen = np.zeros(L, np.int32)
    for r in range(world):
        text, image, image0, shard = mkimage.sp_rows(S, N, world, r)
        assert shard == L // world and text == (S if r == 0 else 0)
        assert text + image == shard
        seen[r * shard:r * shard + text] += 1  # text rows at joint positions 0..S-1
        seen[S + image0:S + image0 + image] += 1
        assert S + image0 == r * shard + text
    assert (seen == 1).all()


@pytest.mark.parametrize("S,N,world", [(256, 4096, 4), (300, 212, 2), (600, 424, 2), (1, 1, 3)])
def test_partition_rejects_unsplittable(S, N, world):
    import mkimage

    with pytest.raises(mkimage.MkbError):
        for r in range(world):
            mkimage.sp_rows(S, N, world, r)


def _exchange_rank(rank, world, port, S, N, B, q):
    import torch
    import torch.distributed as dist
    import mkimage

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        full = np.arange(B * N * 2, dtype=np.float32).reshape(B, N, 2)  # every rank knows the answer
        text, image, image0, Lg = mkimage.sp_rows(S, N, world, rank)
        slot = torch.zeros(B, Lg, 2)
        slot[:, text:] = torch.from_numpy(full[:, image0:image0 + image])  # this rank's velocities, in place
        gathered = [torch.zeros_like(slot) for _ in range(world)]
        dist.all_gather(gathered, slot)
        out = np.zeros_like(full)
        for g in range(world):
            p0, p1 = max(g * Lg, S), (g + 1) * Lg
            if p0 < p1:
                out[:, p0 - S:p1 - S] = gathered[g][:, p0 - g * Lg:].numpy()
        q.put((rank, bool(np.array_equal(out, full))))
    finally:
        dist.destroy_process_group()


def test_velocity_exchange_gloo_world2():
    import multiprocessing as mp
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_exchange_rank, args=(r, 2, port, 128, 384, 3, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    res = dict(q.get(timeout=5) for _ in range(2))
    assert res == {0: True, 1: True}


def _attend(q, k, v):
    s = q @ k.swapaxes(-1, -2) / np.sqrt(q.shape[-1])
    p = np.exp(s - s.max(-1, keepdims=True))
    return (p / p.sum(-1, keepdims=True)) @ v


def _head_exchange_rank(rank, world, port, S, N, B, H, hd, q):
    import torch
    import torch.distributed as dist
    import mkimage

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(11)
        L, Hr = S + N, H // world
        qf, kf, vf = (rng.standard_normal((B, H, L, hd)).astype(np.float32) for _ in range(3))  # every rank knows them
        want = _attend(qf, kf, vf).transpose(0, 2, 1, 3).reshape(B, L, H * hd)  # joint rows, heads side by side
        text, image, image0, Lg = mkimage.sp_rows(S, N, world, rank)
        rows = slice(rank * Lg, (rank + 1) * Lg)
        # The QKV epilogue's send spans: span g = [q|k|v][B][Hr][Lg][hd] of rank g's heads over this rank's rows.
        send = np.stack([np.stack([t[:, g * Hr:(g + 1) * Hr, rows] for t in (qf, kf, vf)]) for g in range(world)])
        recv = torch.empty(send.shape)
        dist.all_to_all_single(recv, torch.from_numpy(np.ascontiguousarray(send, dtype=np.float32)))
        recv = recv.numpy()  # [source rank][q|k|v][B][Hr][Lg][hd]: joint row p is row p % Lg of plane p // Lg
        qa, ka, va = (np.concatenate([recv[g, t] for g in range(world)], axis=2) for t in range(3))
        o = _attend(qa, ka, va)  # [B][Hr][L][hd]: this rank's heads over every joint row
        # Output spans, one per owning rank: [B][Lg][Hr * hd], rows at the owner's local positions.
        osend = np.stack([o[:, :, g * Lg:(g + 1) * Lg].transpose(0, 2, 1, 3).reshape(B, Lg, Hr * hd)
                          for g in range(world)])
        orecv = torch.empty(osend.shape)
        dist.all_to_all_single(orecv, torch.from_numpy(np.ascontiguousarray(osend, dtype=np.float32)))
        mine = np.concatenate(list(orecv.numpy()), axis=2)  # rank g's heads at columns g * Hr * hd
        q.put((rank, bool(np.allclose(mine, want[:, rows], atol=1e-5))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_head_exchange_layout_gloo(world):
    import multiprocessing as mp
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_head_exchange_rank, args=(r, world, port, 128, 896, 2, 8, 16, q))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        if p.is_alive():
            p.kill()
    res = dict(q.get(timeout=5) for _ in range(world))
    assert res == {r: True for r in range(world)}
