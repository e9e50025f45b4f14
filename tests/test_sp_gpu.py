"""Sequence-parallel DiT step (mkb_dit_set_sequence_parallel) on two GPUs against the one-GPU step.

Each rank runs every GEMM, norm and RoPE on its own joint rows and the ranks all-gather K and V per block, so every
output row goes through the same arithmetic in the same order as on one GPU: the bar is bit-for-bit equality of the
velocities and updated latents, on every rank, through the host, guided and device-buffer calls (the guided call
three times: eager, captured into a CUDA graph with the collectives inside, replayed). NVLS is off for these
processes. Skipped with fewer than two GPUs."""

import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

WORKER = os.path.join(os.path.dirname(os.path.abspath(__file__)), "sp_worker.py")


def test_sequence_parallel_two_gpus_bit_exact(tmp_path):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, WORKER, str(r), "2", str(tmp_path)], env=env) for r in range(2)]
    try:
        codes = [p.wait(timeout=300) for p in procs]
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
                p.wait()
    assert codes == [0, 0], codes
    ref = np.load(tmp_path / "ref.npy")
    assert np.isfinite(ref).all() and np.abs(ref).max() > 0
    for r in range(2):
        got = np.load(tmp_path / f"rank{r}.npy")
        assert got.shape == ref.shape
        assert np.array_equal(got, ref), (r, np.abs(got - ref).max())
