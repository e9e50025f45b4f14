"""The GEMM epilogues' two output paths agree bit for bit: tiles staged in shared memory and written by TMA (fp32:
a store, a reduce-add into an in-place residual, or a residual box loaded, added and stored; bf16: a box store)
against per-thread row stores (MKB_TMA_EPI=0, in a child process), for GEMMs, convolutions and GELU projections on
ragged shapes; and the outputs match the oracle (fp32 outputs: max-abs <= 1e-3 of the output scale; bf16: 1e-2)."""

import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def test_add_epilogue_paths_agree(cuda, tmp_path):
    import add_epilogue_cases as cases_mod

    got, status = cases_mod.run(cuda)
    assert status == 0
    path = tmp_path / "thread_stores.npz"
    env = dict(os.environ, MKB_TMA_EPI="0")
    subprocess.run([sys.executable, os.path.join(HERE, "add_epilogue_cases.py"), str(path)], check=True, env=env,
                   timeout=600)
    ref = np.load(path)
    assert int(ref["status"]) == 0
    assert set(ref.files) - {"status"} == set(got)
    for k, v in got.items():
        assert v.shape == ref[k].shape, k
        assert np.array_equal(v.view(np.uint32), ref[k].view(np.uint32)), k


def test_add_epilogue_oracle(cuda):
    from oracle import ops as O
    import add_epilogue_cases as cases_mod

    got, _ = cases_mod.run(cuda)
    for kind, shape, d in cases_mod.inputs("cpu"):
        key = kind + "_" + "x".join(str(s) for s in shape)
        x, w, b = (d[n].float().numpy() for n in ("x", "w", "b"))
        av, r = (d[n].float().numpy() if n in d else None for n in ("av", "r"))
        if kind == "proj":
            ref = O.linear(x, w, b)
            ref = 0.5 * ref * (1.0 + np.tanh(0.7978845608028654 * (ref + 0.044715 * ref ** 3)))
            y = got[f"{key}_gelu"]
            assert np.abs(y - ref).max() < 1e-2 * np.abs(ref).max() + 1e-2, key
            continue
        if kind == "gemm":
            M = shape[0]
            rps = (M + 1) // 2
            base = O.linear(x, w, b)
            avr = av[np.arange(M) // rps]
        else:
            B, H, W, C, Cout, taps, stride = shape
            base = O.conv2d_nhwc(x, w.reshape(Cout, taps, C), stride, taps, b)
            avr = av[:, None, None, :]
        for mode, ref in (("store", base + avr), ("resid", base + r), ("inplace", base + avr + r)):
            err = np.abs(got[f"{key}_{mode}"] - ref).max() / np.abs(ref).max()
            assert err < 1e-3, (key, mode, err)
