"""Failure detection, exercised without faulting the GPU.

* On the device: a GEMM whose first CTA never receives its first stage (mkb_selftest_stalled_gemm) must end on its
  own through the bounded waits, report MKB_ERR_KERNEL through mkb_check_kernels, and leave the context usable.
* On the device, the head exchange's wait for its peers (mkb_selftest_peer_wait): a peer flag that nothing raises
  runs out the bounded wait, is reported as MKB_ERR_KERNEL with the shard-wait bit, and the same wait passes at once
  when every flag is up.
* On the host: an allocation that cannot succeed in mkb_dit_create returns MKB_ERR_ALLOC and leaks nothing; an
  NCCL communicator that cannot be made (a stand-in libnccl bound through MKB_NCCL_LIB whose ncclCommInitRank
  returns an error) makes mkb_dit_set_sequence_parallel fail cleanly, and the handle keeps working on one GPU."""

import ctypes
import os
import subprocess
import sys
import time

import numpy as np
import pytest

from oracle import ops as O
from oracle import qwen_dit as QD
from oracle import rng

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# Status bits: a consumer gave up waiting for a shared-memory stage to fill (1), or the producer for one to be
# released (2). The MMA warp waits on the withheld stage and the producer on its release, each with its own 2 s
# limit, so whichever gives up first reports and the other leaves on the abort flag.
ERR_WAIT_FULL, ERR_WAIT_EMPTY, ERR_WAIT_DRAIN = 1, 2, 16


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def test_stalled_pipeline_times_out_and_context_survives(cuda):
    import torch
    import mkimage

    M, N, K = 256, 512, 512
    g = torch.Generator().manual_seed(3)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).to(cuda)
    w = (0.05 * torch.randn(N, K, generator=g)).to(torch.bfloat16).to(cuda)
    y = torch.zeros(M, N, device=cuda)
    assert mkimage.ops.check_kernels() == 0
    t0 = time.time()
    mkimage.check(mkimage.lib.mkb_selftest_stalled_gemm(_p(x), K, _p(w), K, _p(y), N, M, N, K, None))
    bits = ctypes.c_uint32()
    code = mkimage.lib.mkb_check_kernels(ctypes.byref(bits))  # synchronises: the kernel has returned by now
    elapsed = time.time() - t0
    assert code == 4, (code, mkimage.lib.mkb_last_error())  # MKB_ERR_KERNEL
    assert bits.value & (ERR_WAIT_FULL | ERR_WAIT_EMPTY), hex(bits.value)
    assert bits.value & ERR_WAIT_DRAIN, hex(bits.value)  # the producer's drain gave up on the withheld load
    assert 1.5 < elapsed < 60, elapsed  # two bounded waits of 2 s each, not a hang
    # The status word is cleared and the same context runs the same GEMM correctly.
    assert mkimage.ops.check_kernels() == 0
    got = mkimage.ops.proj(x, w, out_f32=True)
    assert mkimage.ops.check_kernels() == 0
    ref = O.linear(x.float().cpu().numpy(), w.float().cpu().numpy())
    assert np.abs(got.cpu().numpy() - ref).max() <= 1e-4 * np.abs(ref).max()


def _small_cfg(mkimage, **over):
    c = dict(variant=mkimage.QWEN1, hidden=256, heads=2, ffn=512, blocks=1, text_dim=128, max_batch=2,
             max_text_tokens=128, max_image_tokens=128, slots=2)
    c.update(over)
    return mkimage.DitConfig(**c)


def _small_step(mkimage, d):
    D, H, F, NB, TD, h, w, S = 256, 2, 512, 1, 128, 8, 16, 16
    prompt = rng.normal(rng.tensor_key(9, 0), S * TD).reshape(S, TD)
    lat = rng.normal(rng.tensor_key(9, 1), h * w * 64).reshape(h * w, 64)
    d.begin(prompt, h, w, slot=0)
    v = d.step(lat, 0.5, slot=0)
    ref = QD.step(QD.default_cfg("qwen1", D, H, F, NB, TD), d.weights(), lat, prompt, 0.5, h, w)
    rel = float(np.sqrt(((v - ref) ** 2).sum() / (ref ** 2).sum()))
    assert rel < 0.05, rel


def test_dit_create_allocation_failure_leaks_nothing(cuda):
    import torch
    import mkimage

    d = mkimage.Dit(_small_cfg(mkimage))  # the per-device status word and the runtime's own state exist now
    d.close()
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    # 2^28 image tokens: the residual stream alone would need 8 x 2^28 x 256 x 4 bytes (2.2 TB).
    with pytest.raises(mkimage.MkbError) as ei:
        mkimage.Dit(_small_cfg(mkimage, max_batch=8, max_image_tokens=1 << 28))
    assert ei.value.code == 5, ei.value  # MKB_ERR_ALLOC
    assert "allocating" in str(ei.value)
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info()[0]
    assert abs(free1 - free0) < (32 << 20), (free0, free1)
    # No stale error leaks into the next handle's launches.
    d = mkimage.Dit(_small_cfg(mkimage))
    d.init_random(5)
    _small_step(mkimage, d)
    d.close()


_SP_FAIL_CHILD = r"""
import sys
sys.path[:0] = [{root!r}, {pkg!r}]
import torch
import mkimage
from tests.test_failure_gpu import _small_cfg, _small_step

torch.cuda.init()
d = mkimage.Dit(_small_cfg(mkimage))
d.init_random(5)
torch.cuda.synchronize()
free0 = torch.cuda.mem_get_info()[0]
try:
    d.set_sequence_parallel(bytes(128), 0, 2)
    raise SystemExit("set_sequence_parallel succeeded against the failing NCCL")
except mkimage.MkbError as e:
    assert e.code == 2, e  # MKB_ERR_CUDA
    assert "ncclCommInitRank" in str(e) and "injected" in str(e), str(e)
torch.cuda.synchronize()
assert abs(torch.cuda.mem_get_info()[0] - free0) < (32 << 20), "exchange buffers not released"
_small_step(mkimage, d)
d.close()
print("SP_FAIL_OK")
"""


def test_sequence_parallel_nccl_failure_leaves_handle_usable(cuda, tmp_path):
    so = tmp_path / "libfake_nccl.so"
    subprocess.run(["gcc", "-shared", "-fPIC", "-O1", "-o", str(so),
                    os.path.join(ROOT, "tests", "fake_nccl", "fake_nccl.c")], check=True)
    env = dict(os.environ, MKB_NCCL_LIB=str(so))
    code = _SP_FAIL_CHILD.format(root=ROOT, pkg=os.path.join(ROOT, "mako-image_b200"))
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "SP_FAIL_OK" in r.stdout, (r.stdout[-2000:], r.stderr[-4000:])


def test_peer_wait_times_out_and_context_survives(cuda):
    import torch
    import mkimage

    flags = torch.tensor([7, 6, 7, 0], dtype=torch.int64, device=cuda)  # rank 1's flag short; 3 is this rank's own
    value = torch.tensor([7], dtype=torch.int64, device=cuda)
    assert mkimage.ops.check_kernels() == 0
    t0 = time.time()
    mkimage.check(mkimage.lib.mkb_selftest_peer_wait(_p(flags), 4, 3, _p(value), None))
    bits = ctypes.c_uint32()
    code = mkimage.lib.mkb_check_kernels(ctypes.byref(bits))
    elapsed = time.time() - t0
    assert code == 4, (code, mkimage.lib.mkb_last_error())  # MKB_ERR_KERNEL
    assert bits.value == 0x100, hex(bits.value)  # the shard-wait bit
    assert 1.5 < elapsed < 30, elapsed
    flags[1] = 8  # every peer's flag up (at or above the value): no wait, no error
    t0 = time.time()
    mkimage.check(mkimage.lib.mkb_selftest_peer_wait(_p(flags), 4, 3, _p(value), None))
    assert mkimage.ops.check_kernels() == 0
    assert time.time() - t0 < 1.5


def test_exchange_switches_need_sequence_parallelism(cuda):
    """The exchange switches are refused (MKB_ERR_STATE) on a handle without sequence parallelism, which then steps
    normally."""
    import mkimage

    d = mkimage.Dit(_small_cfg(mkimage))
    try:
        d.init_random(5)
        for call, code in ((lambda: mkimage.lib.mkb_dit_sp_head_exchange(d.h, 2), 3),
                           (lambda: mkimage.lib.mkb_dit_sp_head_exchange(d.h, 1), 3),
                           (lambda: mkimage.lib.mkb_dit_sp_peer_exchange(d.h, 1), 3)):
            assert call() == code, mkimage.lib.mkb_last_error()
            assert b"sequence parallelism" in mkimage.lib.mkb_last_error()
        _small_step(mkimage, d)
        assert mkimage.ops.check_kernels() == 0
    finally:
        d.close()
