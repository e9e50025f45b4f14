"""The generation loop's schedule and samplers, restated in Python/numpy.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py). Pinned: the ER-SDE restatement reproduces the reference's own
golden vectors (tests/er_sde_test.cpp:46-56, in tests/golden/er_sde_golden.json) and the reference's er_sde.cpp
compiled here (oracle/_ref, built by oracle/Makefile)."""

import math

import numpy as np


def shift_mu(tokens, base_seq=256.0, max_seq=4096.0, base_shift=0.5, max_shift=1.15, mu=None):
    """Engine::shift_mu (src/image/engine.cpp:335-339)."""
    if mu is not None:
        return mu
    m = (max_shift - base_shift) / (max_seq - base_seq)
    return tokens * m + (base_shift - m * base_seq)


def sigmas(steps, tokens, terminal=0.0, **sched):
    """Engine::sigmas (engine.cpp:347-365): linspace(1, 1/steps) through the exponential time shift, in float,
    optionally stretched to end at `terminal`, then 0."""
    mu = shift_mu(tokens, **sched)
    emu = math.exp(mu)
    s = []
    for i in range(steps):
        t = 1.0 if steps == 1 else float(np.float32(1.0 + (1.0 / steps - 1.0) * i / (steps - 1)))
        s.append(np.float32(emu / (emu + (1.0 / t - 1.0))))
    s = np.array(s, np.float32)
    if terminal > 0 and steps > 0 and s[-1] < 1.0:
        scale = np.float32((np.float32(1.0) - s[-1]) / (np.float32(1.0) - np.float32(terminal)))
        s = (np.float32(1.0) - (np.float32(1.0) - s) / scale).astype(np.float32)
    return np.concatenate([s, np.zeros(1, np.float32)])


def top_sigma(tokens, **sched):
    """Engine::top_sigma (engine.cpp:341-345)."""
    mu = shift_mu(tokens, **sched)
    t = 1 - 1e-4
    return float(np.float32(math.exp(mu) / (math.exp(mu) + (1.0 / t - 1.0))))


def guided_euler(x, v_cond, v_uncond, guidance, sigma, sigma_next):
    """CFG then an Euler step (engine.cpp:476-480, 500-503); returns the new x."""
    v = v_cond if v_uncond is None else v_uncond + np.float32(guidance) * (v_cond - v_uncond)
    return (x + np.float32(sigma_next - sigma) * v).astype(np.float32)


def euler_ancestral(x, v, sigma, sigma_next, noise):
    """Euler-ancestral update of Engine::generate (src/image/engine.cpp:492-499), in place on float32 x: down to the
    level whose noise, with fresh noise of the remainder added, makes the next level's."""
    frm, to = float(sigma), float(sigma_next)
    up = min(to, np.sqrt(to * to * (frm * frm - to * to) / (frm * frm)))
    dt = np.float32(np.sqrt(to * to - up * up) - frm)
    x += dt * np.asarray(v, np.float32)
    if up > 0:
        x += np.float32(up) * np.asarray(noise, np.float32)
    return x


def _scaler(x):
    return x * (math.exp(x ** 0.3) + 10.0)


class ErSde:
    """image::ErSde (src/image/er_sde.cpp:17-74): three-stage ER-SDE with 200-point Riemann sums."""

    POINTS = 200

    def __init__(self, sig, flow, top):
        self.sig = [float(s) for s in sig]
        if len(self.sig) < 2:
            raise ValueError("ER-SDE: no steps")
        if flow and self.sig[0] >= 1:
            self.sig[0] = float(top)
        self.lam = [s / (1 - s) if flow else s for s in self.sig]
        self.old = None
        self.old_d = None

    def sigma(self, i):
        return float(np.float32(self.sig[i]))

    def step(self, i, x, denoised, noise, s_noise=1.0):
        x = np.asarray(x, np.float32)
        den = np.asarray(denoised, np.float32)
        stage = min(3, i + 1)
        if self.sig[i + 1] == 0:
            out = den.copy()
        else:
            ls, lt = self.lam[i], self.lam[i + 1]
            a_s, a_t = self.sig[i] / ls, self.sig[i + 1] / lt
            r = _scaler(lt) / _scaler(ls)
            c1, c2 = a_t / a_s * r, a_t * (1 - r)
            dt = lt - ls
            h = -dt / self.POINTS
            s = su = 0.0
            for k in range(self.POINTS):
                pos = lt + k * h
                sp = _scaler(pos)
                s += 1 / sp
                su += (pos - ls) / sp
            s *= h
            su *= h
            c3 = a_t * (dt + s * _scaler(lt))
            c4 = a_t * (dt * dt / 2 + su * _scaler(lt))
            d_den = ls - self.lam[i - 1] if stage >= 2 else 1.0
            u_den = (ls - self.lam[i - 2]) / 2 if stage >= 3 else 1.0
            cn = a_t * s_noise * math.sqrt(max(0.0, lt * lt - ls * ls * r * r))
            v = c1 * x.astype(np.float64) + c2 * den.astype(np.float64)
            if stage >= 2:
                d = (den.astype(np.float64) - self.old) / d_den
                v = v + c3 * d
                if stage >= 3:
                    v = v + c4 * (d - self.old_d) / u_den
                self.old_d = d.astype(np.float32).astype(np.float64)
            if s_noise > 0:
                v = v + cn * np.asarray(noise, np.float64)
            out = v.astype(np.float32)
        self.old = den.astype(np.float64)
        return out
