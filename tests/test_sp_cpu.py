"""Host logic of the sequence-parallel step, on the CPU.

mkb_dit_sp_rows is the partition the library uses: the shards must tile every sample's joint rows exactly, with all
text rows on rank 0. The velocity exchange (each rank places its image rows at their shard positions, an
all-gather, then every shard's image rows back in token order) is replayed here with a world-size-2 gloo group over
the same partition, so the index arithmetic is checked with a real collective."""

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
