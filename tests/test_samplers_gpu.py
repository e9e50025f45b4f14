"""The device samplers (mkb_euler_ancestral_dev, mkb_er_sde_step_dev, mkb_cfg_combine_dev,
mkb_dit_guided_velocity_dev) against the oracle (oracle/sampler.py, whose ER-SDE reproduces the reference's goldens)
with the same noise: oracle/rng.normal draws the counter-based stream the kernels draw, equal up to libm rounding.

Tolerance: the updates run in float / double like the reference, so per element |device - oracle| <= 1e-5 of the
latents' scale after each step."""

import numpy as np
import pytest

from oracle import rng as R
from oracle import sampler as OS

pytestmark = pytest.mark.gpu


def _t(a, cuda):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(cuda)


def test_euler_ancestral_dev(cuda):
    import mkimage

    rs = np.random.RandomState(1)
    n = 5000
    x = rs.standard_normal(n).astype(np.float32)
    v = rs.standard_normal(n).astype(np.float32)
    key, off = R.tensor_key(7, 3), 123
    for s, s1 in ((0.8, 0.6), (0.3, 0.0), (1.0, 0.999)):
        xd, vd = _t(x, cuda), _t(v, cuda)
        mkimage.euler_ancestral_dev(xd, vd, s, s1, key, off)
        want = OS.euler_ancestral(x.copy(), v, np.float32(s), np.float32(s1), R.normal(key, n, offset=off))
        got = xd.cpu().numpy()
        assert np.abs(got - want).max() <= 1e-5 * max(1.0, np.abs(want).max()), (s, s1)
    with pytest.raises(mkimage.MkbError):
        mkimage.euler_ancestral_dev(_t(x, cuda), _t(v, cuda), 0.5, 0.7, key)  # sigma_next above sigma


@pytest.mark.parametrize("flow", [True, False])
def test_er_sde_dev_run_matches_oracle(cuda, flow):
    import torch
    import mkimage

    steps, n = 6, 4096
    sig = mkimage.sigmas(steps, 256) if flow else np.array([14.6, 8.0, 4.0, 2.0, 1.0, 0.4, 0.0], np.float32)
    top = mkimage.top_sigma(256)
    dev, ref = mkimage.ErSde(sig, flow, top), OS.ErSde(sig, flow, top)
    rs = np.random.RandomState(2)
    x = (rs.standard_normal(n) * (1.0 if flow else 14.6)).astype(np.float32)
    xd = _t(x, cuda)
    state = torch.zeros(2 * n, device=cuda)
    key = R.tensor_key(9, 0)
    for i in range(steps):
        v = rs.standard_normal(n).astype(np.float32)
        s_i = np.float32(ref.sigma(i))
        dev.step_dev(i, xd, _t(v, cuda), state, key, noise_offset=i * n)
        den = (x - s_i * v).astype(np.float32)  # the image estimate (engine.cpp:483-486)
        noise = R.normal(key, n, offset=i * n) if sig[i + 1] > 0 else None
        x = ref.step(i, x, den, noise)
        got = xd.cpu().numpy()
        assert np.abs(got - x).max() <= 1e-5 * max(1.0, np.abs(x).max()), (flow, i)
    with pytest.raises(mkimage.MkbError, match="0, 1, 2"):
        dev.step_dev(3, xd, _t(v, cuda), state, key)  # not the next step of a run


def test_guided_velocity_dev(cuda):
    import torch
    import mkimage

    cfg = mkimage.DitConfig(variant=mkimage.QWEN1, hidden=256, heads=2, ffn=512, blocks=2, text_dim=256, max_batch=4,
                            max_text_tokens=16, max_image_tokens=96, slots=4)
    d = mkimage.Dit(cfg)
    d.init_random(seed=3)
    rs = np.random.RandomState(4)
    for s in range(4):
        d.begin(rs.standard_normal((16, 256)).astype(np.float32), 8, 12, slot=s)
    N = 96
    lat = _t(rs.standard_normal((2, N, 64)), cuda)
    v = torch.empty_like(lat)
    d.guided_velocity_dev(2, lat.data_ptr(), 0.7, 3.5, v.data_ptr())
    raw = torch.empty(4, N, 64, device=cuda)
    d.step_batch_dev([0, 1, 2, 3], torch.stack([lat[0], lat[0], lat[1], lat[1]]).contiguous().data_ptr(),
                     [0.7] * 4, raw.data_ptr())
    torch.cuda.synchronize()
    r = raw.cpu().numpy()
    want = np.stack([r[1] + np.float32(3.5) * (r[0] - r[1]), r[3] + np.float32(3.5) * (r[2] - r[3])])
    got = v.cpu().numpy()
    assert np.abs(got - want).max() <= 1e-5 * max(1.0, np.abs(want).max())
    assert mkimage.ops.check_kernels() == 0
