"""The C++ Engine mirror (mako-image_b200/host/engine.hpp) through its own C++ test programs (tests/cpp/)."""

import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "mako-image_b200")


def _build_and_run(name):
    subprocess.run(["make", "-C", PKG, "-s", "tests"], check=True, capture_output=True)
    r = subprocess.run([os.path.join(PKG, "build", name)], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr


def test_engine_loop_cpu():
    """Schedule, guided Euler and ER-SDE loops over a made-up model (no GPU)."""
    _build_and_run("engine_cpu_test")


@pytest.mark.gpu
def test_engine_guided_steps_gpu(cuda):
    """Engine::denoise's batched guided steps on the device against unbatched step() calls, both DiT variants and the
    SDXL UNet, and the VAE decode, all through the C ABI."""
    _build_and_run("engine_gpu_test")
