"""The schedule and samplers: the oracle's ER-SDE against the reference's golden vectors and the reference's own
er_sde.cpp (compiled into oracle/_ref when the reference tree was present at build time), and the library's C++
sampler (mkb_er_sde_*, mkb_sigmas, mkb_guided_euler) against both. CPU only."""

import ctypes
import json
import math
import os

import numpy as np
import pytest

from oracle import sampler as OS

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLD = json.load(open(os.path.join(ROOT, "tests", "golden", "er_sde_golden.json")))
REF_SO = os.path.join(ROOT, "oracle", "_ref", "liber_sde_ref.so")


def _model(x, s, j):
    # the made-up model of the reference's test (er_sde_test.cpp:22-26)
    return np.tanh(x * (0.6 + 0.2 * s)) + 0.1 * np.cos(j + 3 * s)


def _run(make, sched, flow, top, s_noise):
    n = GOLD["n"]
    sig = np.array(sched, np.float32)
    er = make(sig, flow, top)
    j = np.arange(n)
    x = (np.sin(1.7 * j + 0.3) * sig[0]).astype(np.float32)
    for i in range(len(sig) - 1):
        s = er.sigma(i)
        d = _model(x, np.float32(s), j).astype(np.float32)
        noise = np.sin(0.9 * j + 1.3 * (i + 1)).astype(np.float32)
        x = er.step(i, x, d, noise, s_noise) if isinstance(er, OS.ErSde) else _lib_step(er, i, x, d, noise, s_noise)
    return x


def _lib_step(er, i, x, d, noise, s_noise):
    x = x.copy()
    er.step(i, x, d, noise, s_noise)
    return x


def _rel(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return float(np.sqrt(((got - want) ** 2).sum() / (want ** 2).sum()))


@pytest.mark.parametrize("case", GOLD["cases"], ids=[c["name"] for c in GOLD["cases"]])
def test_oracle_er_sde_golden(case):
    x = _run(OS.ErSde, GOLD["schedules"][case["schedule"]], case["flow"], GOLD["top"], case["s_noise"])
    assert _rel(x, case["want"]) < GOLD["tolerance_rel"]


@pytest.mark.parametrize("case", GOLD["cases"], ids=[c["name"] for c in GOLD["cases"]])
def test_library_er_sde_golden(case):
    import mkimage

    x = _run(mkimage.ErSde, GOLD["schedules"][case["schedule"]], case["flow"], GOLD["top"], case["s_noise"])
    assert _rel(x, case["want"]) < GOLD["tolerance_rel"]
    y = _run(OS.ErSde, GOLD["schedules"][case["schedule"]], case["flow"], GOLD["top"], case["s_noise"])
    assert np.abs(x - y).max() <= 1e-6 * max(1.0, np.abs(y).max())


class _RefErSde:
    lib = None

    def __init__(self, sig, flow, top):
        L = _RefErSde.lib
        self.sig = np.ascontiguousarray(sig, np.float32)
        self.h = L.ref_er_sde_create(self.sig.ctypes.data_as(ctypes.c_void_p), len(sig), int(flow), top)

    def sigma(self, i):
        return _RefErSde.lib.ref_er_sde_sigma(self.h, i)

    def step(self, i, x, d, noise, s_noise):
        """In place, like the library's binding."""
        _RefErSde.lib.ref_er_sde_step(self.h, i, x.ctypes.data_as(ctypes.c_void_p), d.ctypes.data_as(ctypes.c_void_p),
                                      noise.ctypes.data_as(ctypes.c_void_p), len(x), s_noise)


@pytest.mark.skipif(not os.path.exists(REF_SO), reason="reference er_sde.cpp not built (oracle/Makefile)")
@pytest.mark.parametrize("case", GOLD["cases"], ids=[c["name"] for c in GOLD["cases"]])
def test_reference_er_sde_matches_oracle(case):
    L = ctypes.CDLL(REF_SO)
    L.ref_er_sde_create.restype = ctypes.c_void_p
    L.ref_er_sde_create.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_float]
    L.ref_er_sde_sigma.restype = ctypes.c_float
    L.ref_er_sde_sigma.argtypes = [ctypes.c_void_p, ctypes.c_int]
    L.ref_er_sde_step.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                  ctypes.c_long, ctypes.c_float]
    _RefErSde.lib = L
    got_ref = _run(lambda s, f, t: _RefErSde(s, f, t), GOLD["schedules"][case["schedule"]], case["flow"], GOLD["top"],
                   case["s_noise"])
    got_or = _run(OS.ErSde, GOLD["schedules"][case["schedule"]], case["flow"], GOLD["top"], case["s_noise"])
    assert np.abs(got_ref - got_or).max() <= 1e-6 * max(1.0, np.abs(got_or).max())
    assert _rel(got_ref, case["want"]) < GOLD["tolerance_rel"]


@pytest.mark.parametrize("steps,tokens,terminal", [(40, 4096, 0.0), (28, 1024, 0.0), (8, 16384, 0.02), (1, 256, 0.0),
                                                   (20, 64, 0.1)])
def test_sigmas_library_vs_oracle(steps, tokens, terminal):
    import mkimage

    sch = mkimage.Schedule.default()
    sch.terminal = terminal
    got = mkimage.sigmas(steps, tokens, sch)
    want = OS.sigmas(steps, tokens, terminal=terminal)
    assert got.shape == (steps + 1,) and got[-1] == 0
    assert np.abs(got - want).max() <= 1e-6
    assert np.all(np.diff(got) <= 0)  # decreasing to 0
    assert abs(mkimage.top_sigma(tokens) - OS.top_sigma(tokens)) < 1e-7


def test_sigmas_known_values():
    import mkimage

    # shift mu at 4096 tokens is max_shift = 1.15; the first level is exactly 1, the last before 0 is
    # e^mu / (e^mu + steps - 1) at t = 1/steps.
    s = mkimage.sigmas(40, 4096)
    assert s[0] == 1.0
    assert abs(s[39] - math.exp(1.15) / (math.exp(1.15) + 39.0)) < 1e-6


def test_guided_euler_library_vs_oracle():
    import mkimage

    r = np.random.default_rng(0)
    x, vc, vu = (r.standard_normal(1000).astype(np.float32) for _ in range(3))
    want = OS.guided_euler(x, vc, vu, 4.0, 0.7, 0.6)
    got = x.copy()
    mkimage.guided_euler(got, vc, vu, 4.0, 0.7, 0.6)
    assert np.abs(got - want).max() < 1e-6
