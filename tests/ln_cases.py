"""The ln_modulate cases of tests/test_ln_gpu.py: row widths covering every kernel instance (n 640, 1280, 3072,
4096), ragged row counts, the split between two modulation rows, with and without a shift."""

CASES = [(8192, 3072, 0, True), (700, 3072, 256, True), (37, 640, 5, False), (4099, 1280, 0, True),
         (300, 4096, 100, False)]


def inputs(dev):
    import torch

    g = torch.Generator().manual_seed(77)
    out = []
    for rows, n, split, with_shift in CASES:
        x = (torch.randn(rows, n, generator=g) * 2.0 + 0.5).to(dev)
        mod = (torch.randn(2, n, generator=g) * 0.3).to(dev)
        shift = (torch.randn(2, n, generator=g) * 0.3).to(dev) if with_shift else None
        out.append(((rows, n, split, with_shift), x, mod, shift))
    return out


def run(dev):
    import mkimage

    res = {}
    for (rows, n, split, ws), x, mod, shift in inputs(dev):
        y = mkimage.ops.ln_modulate(x, mod, shift, eps=1e-6, split=split, mod_stride=n, mod_off=0)
        res[f"ln_{rows}x{n}_{split}_{int(ws)}"] = y.float().cpu().numpy()
    return res, mkimage.ops.check_kernels()

