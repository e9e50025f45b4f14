"""One process driving two devices: each kernel's shared-memory limit must be raised on every device it runs on.

GroupNorm at C = 6144 needs 49156 bytes of dynamic shared memory (above the 48 KB default) and every tcgen05 GEMM
more than 100 KB; both run on device 0 and then on device 1 of the same process and must match the oracle there
too (the limit is a per-device setting of the kernel, not a per-process one)."""

import numpy as np
import pytest

from oracle import ops as O

pytestmark = pytest.mark.gpu


def test_group_norm_and_gemm_on_two_devices_in_one_process(cuda):
    import torch

    import mkimage

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    B, HW, C, M, N, K = 1, 256, 6144, 300, 512, 320
    rs = np.random.RandomState(5)
    x = rs.randn(B, HW, C).astype(np.float32)
    g = (1 + 0.1 * rs.randn(C)).astype(np.float32)
    b = (0.1 * rs.randn(C)).astype(np.float32)
    a = O.bf16_round(rs.randn(M, K).astype(np.float32))
    w = O.bf16_round(0.05 * rs.randn(N, K).astype(np.float32))
    want_gn = O.group_norm_nhwc(x, g, b, 32, 1e-5, True)
    want_mm = O.linear(a, w)
    prev = torch.cuda.current_device()
    try:
        for dev in (0, 1):
            torch.cuda.set_device(dev)
            d = torch.device("cuda", dev)
            y = mkimage.ops.group_norm(torch.from_numpy(x).to(d), torch.from_numpy(g).to(d), torch.from_numpy(b).to(d),
                                       groups=32, eps=1e-5, silu=True)
            mm = mkimage.ops.proj(torch.from_numpy(a).to(d).bfloat16(), torch.from_numpy(w).to(d).bfloat16(),
                                  out_f32=True)
            torch.cuda.synchronize(d)
            got_gn = y.float().cpu().numpy()
            assert np.abs(got_gn - want_gn).max() <= 2e-2 * max(1.0, np.abs(want_gn).max()), dev
            assert np.abs(mm.cpu().numpy() - want_mm).max() <= 1e-3 * max(1.0, np.abs(want_mm).max()), dev
            assert mkimage.ops.check_kernels() == 0
    finally:
        torch.cuda.set_device(prev)
