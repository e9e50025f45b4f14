"""The epilogue cases shared by tests/test_add_epilogue_gpu.py and its child process: fp32-output GEMMs and
convolutions with and without a residual (in place and out of place) and a per-sample addvec, and bf16 GELU
projections, on ragged shapes.

Run as a script (`python tests/add_epilogue_cases.py out.npz`) it computes every case on cuda:0 and saves the
outputs, so a process started with another environment (MKB_TMA_EPI=0) can be compared bit for bit."""

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

GEMMS = [(700, 640, 320), (2048, 1280, 1280), (300, 96, 64), (8192, 640, 640)]
# bf16 projections with the tanh-GELU: 128-wide pair tiles, 64-wide tiles with a partial last box, many-tile
# 256-wide pairs (bf16 TMA boxes), and 160-wide tiles (per-thread stores).
PROJS = [(700, 640, 320), (300, 96, 64), (4096, 3072, 1024), (2048, 1280, 1280)]
CONVS = [(2, 16, 32, 64, 96, 9, 1), (1, 24, 16, 64, 256, 9, 1), (1, 12, 8, 64, 64, 9, 1), (1, 32, 32, 128, 64, 9, 2)]


def inputs(dev):
    """Seeded inputs of every case (created on the CPU, so both processes see the same values)."""
    import torch

    g = torch.Generator().manual_seed(1234)

    def t(*shape, scale=1.0):
        return (torch.randn(*shape, generator=g) * scale).to(dev)

    cases = []
    for M, N, K in GEMMS:
        cases.append(("gemm", (M, N, K), dict(x=t(M, K).to(torch.bfloat16), w=t(N, K, scale=0.05).to(torch.bfloat16),
                                              b=t(N, scale=0.1), av=t(2, N, scale=0.1), r=t(M, N))))
    for M, N, K in PROJS:
        cases.append(("proj", (M, N, K), dict(x=t(M, K).to(torch.bfloat16), w=t(N, K, scale=0.05).to(torch.bfloat16),
                                              b=t(N, scale=0.1))))
    for B, H, W, C, Cout, taps, stride in CONVS:
        Ho, Wo = (H - 1) // stride + 1, (W - 1) // stride + 1
        cases.append(("conv", (B, H, W, C, Cout, taps, stride),
                      dict(x=t(B, H, W, C).to(torch.bfloat16), w=t(Cout, taps * C, scale=0.05).to(torch.bfloat16),
                           b=t(Cout, scale=0.1), av=t(B, Cout, scale=0.1), r=t(B, Ho, Wo, Cout))))
    return cases


def run(dev):
    """Every case's outputs: {name: float32 numpy array}. Modes: no residual, residual into a new output, in place."""
    import mkimage

    out = {}
    for kind, shape, d in inputs(dev):
        key = kind + "_" + "x".join(str(s) for s in shape)
        if kind == "proj":
            out[key + "_gelu"] = mkimage.ops.proj(d["x"], d["w"], d["b"], act=mkimage.ops.ACT_GELU_TANH)
            continue
        if kind == "gemm":
            M = shape[0]
            rps = (M + 1) // 2
            out[key + "_store"] = mkimage.ops.proj_add(d["x"], d["w"], d["b"], addvec=d["av"], rows_per_sample=rps)
            out[key + "_resid"] = mkimage.ops.proj_add(d["x"], d["w"], d["b"], resid=d["r"])
            r = d["r"].clone()
            mkimage.ops.proj_add(d["x"], d["w"], d["b"], addvec=d["av"], rows_per_sample=rps, resid=r, out=r)
            out[key + "_inplace"] = r
        else:
            taps, stride = shape[5], shape[6]
            out[key + "_store"] = mkimage.ops.conv2d(d["x"], d["w"], taps=taps, stride=stride, bias=d["b"],
                                                     addvec=d["av"])
            out[key + "_resid"] = mkimage.ops.conv2d(d["x"], d["w"], taps=taps, stride=stride, bias=d["b"],
                                                     resid=d["r"])
            r = d["r"].clone()
            mkimage.ops.conv2d(d["x"], d["w"], taps=taps, stride=stride, bias=d["b"], addvec=d["av"], resid=r, out=r)
            out[key + "_inplace"] = r
    status = mkimage.ops.check_kernels()
    return {k: v.float().cpu().numpy() for k, v in out.items()}, status


if __name__ == "__main__":
    for p in (ROOT, os.path.join(ROOT, "mako-image_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import numpy as np
    import torch

    res, st = run(torch.device("cuda:0"))
    np.savez(sys.argv[1], status=np.array(st), **res)
