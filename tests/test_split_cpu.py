"""The sample-split benchmark mode's CFG pair exchange (bench.py cfg_pair_group) on CPU with gloo, world size 4:
ranks 2i (cond) and 2i + 1 (uncond) all-gather their predictions within their pair and both form the same guided
velocity v_u + g (v_c - v_u), without seeing the other pair's."""

import os

import pytest
import torch
import torch.multiprocessing as mp


def _worker(rank, ws, port, out):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.distributed.init_process_group("gloo", rank=rank, world_size=ws)
    import bench

    grp = bench.cfg_pair_group(torch.distributed, ws, rank)
    vel = torch.full((6,), float(rank + 1))
    both = [torch.empty(6), torch.empty(6)]
    torch.distributed.all_gather(both, vel, group=grp)
    guided = both[1] + 4.0 * (both[0] - both[1])
    out[rank] = guided.tolist()
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()


def test_cfg_pair_exchange_gloo():
    ws = 4
    port = 29600 + os.getpid() % 1000
    with mp.Manager() as m:
        out = m.dict()
        mp.spawn(_worker, args=(ws, port, out), nprocs=ws, join=True)
        res = dict(out)
    for r in range(ws):
        c, u = float(r - r % 2 + 1), float(r - r % 2 + 2)  # values of the pair's even and odd rank
        assert res[r] == pytest.approx([u + 4.0 * (c - u)] * 6)
