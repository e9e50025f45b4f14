"""Schedule and samplers of the generation loop (include/mkb_image.h, schedule section)."""

import ctypes

import numpy as np

from ._lib import lib, check, stream_ptr


class Schedule(ctypes.Structure):
    _fields_ = [("base_seq", ctypes.c_double), ("max_seq", ctypes.c_double), ("base_shift", ctypes.c_double),
                ("max_shift", ctypes.c_double), ("terminal", ctypes.c_double), ("fixed_mu", ctypes.c_int),
                ("mu", ctypes.c_double)]

    @classmethod
    def default(cls):
        s = cls()
        lib.mkb_schedule_default(ctypes.byref(s))
        return s


def _f(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def sigmas(steps, tokens, schedule=None):
    out = np.empty(steps + 1, np.float32)
    check(lib.mkb_sigmas(ctypes.byref(schedule) if schedule else None, steps, tokens, _f(out)))
    return out


def top_sigma(tokens, schedule=None):
    return lib.mkb_top_sigma(ctypes.byref(schedule) if schedule else None, tokens)


def guided_euler(x, v_cond, v_uncond, guidance, sigma, sigma_next):
    """In place on float32 numpy arrays."""
    lib.mkb_guided_euler(_f(x), _f(v_cond), _f(v_uncond) if v_uncond is not None else None, guidance, sigma,
                         sigma_next, x.size)


class ErSde:
    def __init__(self, sig, flow, top):
        s = np.ascontiguousarray(sig, np.float32)
        h = ctypes.c_void_p()
        check(lib.mkb_er_sde_create(_f(s), len(s), int(flow), top, ctypes.byref(h)))
        self.h = h

    def __del__(self):
        if getattr(self, "h", None):
            lib.mkb_er_sde_destroy(self.h)
            self.h = None

    def sigma(self, i):
        return lib.mkb_er_sde_sigma(self.h, i)

    def step_dev(self, i, x, v, state, noise_key, noise_offset=0, s_noise=1.0):
        """The device step on torch CUDA float32 tensors (mkb_er_sde_step_dev): x updated in place from the guided
        model output v; state: 2 * x.numel() floats kept across the run's steps."""
        check(lib.mkb_er_sde_step_dev(self.h, i, x.data_ptr(), v.data_ptr(), state.data_ptr(), noise_key,
                                      noise_offset, x.numel(), s_noise, stream_ptr()))

    def step(self, i, x, denoised, noise, s_noise=1.0):
        """x updated in place (float32 numpy)."""
        d = np.ascontiguousarray(denoised, np.float32)
        nz = np.ascontiguousarray(noise, np.float32) if noise is not None else None
        check(lib.mkb_er_sde_step(self.h, i, _f(x), _f(d), _f(nz) if nz is not None else None, x.size, s_noise))


def cfg_combine_dev(out, v_cond, v_uncond, guidance):
    """out = v_uncond + guidance (v_cond - v_uncond) on torch CUDA float32 tensors."""
    check(lib.mkb_cfg_combine_dev(out.data_ptr(), v_cond.data_ptr(), v_uncond.data_ptr(), guidance, out.numel(),
                                  stream_ptr()))


def euler_ancestral_dev(x, v, sigma, sigma_next, noise_key, noise_offset=0):
    """The Euler-ancestral update of device latents x (torch CUDA float32) from the guided velocity v."""
    check(lib.mkb_euler_ancestral_dev(x.data_ptr(), v.data_ptr(), sigma, sigma_next, noise_key, noise_offset, x.numel(),
                                      stream_ptr()))
