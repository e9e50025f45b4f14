"""The seeded synthetic-input generator shared by the oracle and the CUDA library (mkb_fill_normal).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py). Counter-based: element i of a tensor with key k is produced from
splitmix64(k + i // 2) by the Box-Muller transform (even i: cos branch, odd i: sin branch), so any slice can be
generated independently and the device kernel produces the same values (up to libm rounding)."""

import numpy as np

_M64 = (1 << 64) - 1
GOLDEN = 0x9E3779B97F4A7C15


def splitmix64(x):
    """SplitMix64 finaliser of (x + golden gamma), on numpy uint64 arrays or Python ints."""
    if isinstance(x, (int, np.integer)):
        z = (int(x) + GOLDEN) & _M64
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
        return z ^ (z >> 31)
    with np.errstate(over="ignore"):
        z = x.astype(np.uint64) + np.uint64(GOLDEN)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def tensor_key(seed, index):
    """The key of the index-th tensor drawn from a seed."""
    return splitmix64((int(seed) * 0x100000001B3 + int(index)) & _M64)


def normal(key, n, std=1.0, mean=0.0, offset=0):
    """n normals (fp32) of the stream `key`, starting at element `offset`."""
    i = np.arange(offset, offset + n, dtype=np.uint64)
    with np.errstate(over="ignore"):
        h = splitmix64(np.uint64(key) + (i >> np.uint64(1)))
    u1 = ((h >> np.uint64(40)).astype(np.float64) + 0.5) / 16777216.0
    u2 = (h & np.uint64(0xFFFFFF)).astype(np.float64) / 16777216.0
    r = np.sqrt(-2.0 * np.log(u1))
    ang = 2.0 * np.pi * u2
    z = np.where((i & np.uint64(1)) == 0, r * np.cos(ang), r * np.sin(ang))
    return (z * std + mean).astype(np.float32)
