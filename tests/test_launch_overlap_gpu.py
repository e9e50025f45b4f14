"""Programmatic dependent launch changes no result: every kernel waits for its predecessor before touching global
memory, so a DiT step, a UNet step (eager, captured and replayed) and a VAE decode give the same bits with the
launch attribute (this process) and without it (MKB_PDL=0, in a child process)."""

import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def test_launch_overlap_changes_no_bits(cuda, tmp_path):
    import launch_cases

    got, status = launch_cases.run()
    assert status == 0
    path = tmp_path / "no_pdl.npz"
    subprocess.run([sys.executable, os.path.join(HERE, "launch_cases.py"), str(path)], check=True,
                   env=dict(os.environ, MKB_PDL="0"), timeout=600)
    ref = np.load(path)
    assert int(ref["status"]) == 0
    assert set(ref.files) - {"status"} == set(got)
    for k, v in got.items():
        assert np.isfinite(v).all() and np.abs(v).max() > 0, k
        assert np.array_equal(v.view(np.uint32), ref[k].view(np.uint32)), k
