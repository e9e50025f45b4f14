"""One rank of the two-GPU sequence-parallel test (test_sp_gpu.py), run as its own process.

Rank 0 makes the NCCL id and hands it to the other ranks through a file in the shared temporary folder. Every rank
runs the same steps on a sequence-parallel handle, its K/V exchanged by the NCCL all-gather, (argument "peer") by
pushes into the peers' memory, or by the head-parallel exchange over NCCL (argument "heads") or over peer memory
("heads_peer"); rank 0 also runs them on an unsplit handle as the reference. Results go to
rank<r>.npy / ref.npy in that folder."""

import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "mako-image_b200"))

S, GH, GW, TD = 128, 16, 24, 256  # L = 512: two shards of 256 rows, all text rows on rank 0


def run_steps(d, lat):
    """Per-slot velocity, then the guided step three times (eager, graph capture, replay), then the device path."""
    import torch

    out = [d.step(lat, 0.7, slot=1)]
    x = lat
    for _ in range(3):
        x = d.step_cfg(x, 0.7, 0.5, 4.0)
        out.append(x)
    xd = torch.from_numpy(np.stack([lat, -lat])).cuda()
    d.step_cfg_dev(2, xd.data_ptr(), 0.6, 0.45, 3.0)
    torch.cuda.synchronize()
    out.extend(xd.cpu().numpy())
    return np.stack(out)


def main():
    rank, world, tmp = int(sys.argv[1]), int(sys.argv[2]), sys.argv[3]
    exchange = sys.argv[4] if len(sys.argv) > 4 else "nccl"
    wide = len(sys.argv) > 5 and sys.argv[5] == "wide"  # Qwen-Image's widths, 2 blocks, 1024^2 (L = 4352)
    import torch
    import mkimage

    torch.cuda.set_device(rank)
    global S, GH, GW, TD
    if wide:
        S, GH, GW, TD = 256, 64, 64, 3584
        cfg = mkimage.DitConfig(variant=mkimage.QWEN1, hidden=3072, heads=24, ffn=12288, blocks=2, text_dim=TD,
                                max_batch=4, max_text_tokens=S, max_image_tokens=GH * GW, slots=4)
    else:
        cfg = mkimage.DitConfig(variant=mkimage.QWEN1, hidden=256, heads=2, ffn=512, blocks=2, text_dim=TD,
                                max_batch=4, max_text_tokens=S, max_image_tokens=GH * GW, slots=4)
    idf = os.path.join(tmp, "nccl_id")
    if rank == 0:
        nid = mkimage.nccl_unique_id()
        with open(idf + ".part", "wb") as f:
            f.write(nid)
        os.replace(idf + ".part", idf)
    else:
        t0 = time.time()
        while not os.path.exists(idf):
            if time.time() - t0 > 120:
                raise SystemExit("no NCCL id from rank 0")
            time.sleep(0.05)
        with open(idf, "rb") as f:
            nid = f.read()
    rng = np.random.RandomState(7)
    prompts = rng.standard_normal((4, S, TD)).astype(np.float32)
    lat = rng.standard_normal((GH * GW, 64)).astype(np.float32)

    def make(sp):
        d = mkimage.Dit(cfg)
        d.init_random(seed=5)
        if sp:
            d.set_sequence_parallel(nid, rank, world)
            if exchange == "peer":
                d.set_peer_exchange(True)
            elif exchange == "heads":
                d.set_head_exchange(1)
            elif exchange == "heads_peer":
                d.set_head_exchange(2)
        for slot in range(4):
            d.begin(prompts[slot], GH, GW, slot)
        return d

    d = make(True)
    np.save(os.path.join(tmp, f"rank{rank}.npy"), run_steps(d, lat))
    assert mkimage.ops.check_kernels() == 0
    d.close()
    if rank == 0:
        ref = make(False)
        np.save(os.path.join(tmp, "ref.npy"), run_steps(ref, lat))
        ref.close()


if __name__ == "__main__":
    main()
