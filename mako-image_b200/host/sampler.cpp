// The denoising schedule and samplers of the reference's generation loop (src/image/engine.cpp:335-506 and
// src/image/er_sde.cpp), restated for the C ABI: the shifted flow-matching schedule, the guided Euler update and the
// ER-SDE solver. Host code; the guided Euler update also runs fused on the device (mkb_dit_step_cfg).
#include "../../include/mkb_image.h"
#include "er_sde_coef.hpp"

#include <algorithm>
#include <cmath>
#include <new>
#include <vector>

namespace {

double shift_mu(const mkb_schedule& s, uint32_t tokens)
{
    // engine.cpp:335-339: mu linear in the token count between (base_seq, base_shift) and (max_seq, max_shift),
    // unless the model fixes it.
    if (s.fixed_mu)
        return s.mu;
    const double m = (s.max_shift - s.base_shift) / (s.max_seq - s.base_seq);
    return double(tokens) * m + (s.base_shift - m * s.base_seq);
}

// x * (exp(x^0.3) + 10): the ER-SDE noise scaler (er_sde.cpp:11).
double er_scaler(double x) { return x * (std::exp(std::pow(x, 0.3)) + 10.0); }

}  // namespace

struct mkb_er_sde {
    std::vector<double> sigmas, lambdas;
    std::vector<float> old, old_d;
    bool have_old = false, have_old_d = false;
    int dev_next = 0;  // the device step expected next (its state lives in the caller's device buffer)
};

extern "C" {

void mkb_schedule_default(mkb_schedule* s)
{
    if (!s)
        return;
    s->base_seq = 256;
    s->max_seq = 4096;
    s->base_shift = 0.5;
    s->max_shift = 1.15;
    s->terminal = 0;
    s->fixed_mu = 0;
    s->mu = 0;
}

mkb_status mkb_sigmas(const mkb_schedule* sched, uint32_t steps, uint32_t tokens, float* out)
{
    mkb_schedule def;
    mkb_schedule_default(&def);
    const mkb_schedule& s = sched ? *sched : def;
    if (!out || steps == 0)
        return MKB_ERR_INVALID;
    const double mu = shift_mu(s, tokens), emu = std::exp(mu);
    // linspace(1, 1/steps, steps), then exp(mu) / (exp(mu) + 1/t - 1) in float (engine.cpp:353-357).
    for (uint32_t i = 0; i < steps; ++i) {
        const float t = steps == 1 ? 1.0f : float(1.0 + (1.0 / steps - 1.0) * double(i) / double(steps - 1));
        out[i] = float(emu / (emu + (1.0 / double(t) - 1.0)));
    }
    // Stretched to end at the terminal level, unless the last level is 1 (engine.cpp:359-363).
    if (s.terminal > 0 && out[steps - 1] < 1.0f) {
        const float scale = (1.0f - out[steps - 1]) / (1.0f - float(s.terminal));
        for (uint32_t i = 0; i < steps; ++i)
            out[i] = 1.0f - (1.0f - out[i]) / scale;
    }
    out[steps] = 0.0f;
    return MKB_OK;
}

float mkb_top_sigma(const mkb_schedule* sched, uint32_t tokens)
{
    mkb_schedule def;
    mkb_schedule_default(&def);
    const double mu = shift_mu(sched ? *sched : def, tokens), t = 1 - 1e-4;
    return float(std::exp(mu) / (std::exp(mu) + (1.0 / t - 1.0)));  // engine.cpp:341-345
}

void mkb_guided_euler(float* x, const float* v_cond, const float* v_uncond, float guidance, float sigma,
                      float sigma_next, long n)
{
    // v = neg + scale (pos - neg); x += (sigma_next - sigma) v (engine.cpp:476-480, 500-503).
    const float dt = sigma_next - sigma;
    for (long j = 0; j < n; ++j) {
        const float v = v_uncond ? v_uncond[j] + guidance * (v_cond[j] - v_uncond[j]) : v_cond[j];
        x[j] += dt * v;
    }
}

mkb_status mkb_er_sde_create(const float* sigmas, int n, int flow, float top, mkb_er_sde** out)
{
    if (!sigmas || n < 2 || !out)
        return MKB_ERR_INVALID;
    auto* e = new (std::nothrow) mkb_er_sde;
    if (!e)
        return MKB_ERR_ALLOC;
    e->sigmas.assign(sigmas, sigmas + n);
    // A flow model's first level of 1 has no image left to scale: start from `top` (er_sde.cpp:20-22).
    if (flow && e->sigmas[0] >= 1)
        e->sigmas[0] = top;
    for (double s : e->sigmas)
        e->lambdas.push_back(flow ? s / (1 - s) : s);
    *out = e;
    return MKB_OK;
}

void mkb_er_sde_destroy(mkb_er_sde* e) { delete e; }

float mkb_er_sde_sigma(const mkb_er_sde* e, int i)
{
    return e && i >= 0 && i < int(e->sigmas.size()) ? float(e->sigmas[i]) : -1.0f;
}

mkb_status mkb_er_sde_step(mkb_er_sde* e, int i, float* x, const float* denoised, const float* noise, long n,
                           float s_noise)
{
    if (!e || !x || !denoised || i < 0 || i + 1 >= int(e->sigmas.size()) || n <= 0)
        return MKB_ERR_INVALID;
    if ((e->have_old && long(e->old.size()) != n))
        return MKB_ERR_INVALID;
    mkb::ErSdeCoef c;
    mkb::er_sde_coef(e, i, s_noise, &c);
    if (c.last) {
        // The last step lands on the model's image (er_sde.cpp:33-34).
        std::copy(denoised, denoised + n, x);
    } else {
        if (!noise && s_noise > 0)
            return MKB_ERR_INVALID;
        if ((c.stage >= 2 && !e->have_old) || (c.stage >= 3 && !e->have_old_d))
            return MKB_ERR_STATE;
        std::vector<float> dd(c.stage >= 2 ? n : 0);
        for (long j = 0; j < n; ++j) {
            double v = c.c1 * x[j] + c.c2 * denoised[j];
            if (c.stage >= 2) {
                const double d = (double(denoised[j]) - e->old[j]) / c.d_den;
                dd[j] = float(d);
                v += c.c3 * d;
                if (c.stage >= 3)
                    v += c.c4 * (d - e->old_d[j]) / c.u_den;
            }
            if (s_noise > 0)
                v += c.cn * noise[j];
            x[j] = float(v);
        }
        if (c.stage >= 2) {
            e->old_d = std::move(dd);
            e->have_old_d = true;
        }
    }
    e->old.assign(denoised, denoised + n);
    e->have_old = true;
    return MKB_OK;
}

}  // extern "C"

namespace mkb {

bool er_sde_coef(const mkb_er_sde* e, int i, float s_noise, ErSdeCoef* c)
{
    if (!e || i < 0 || i + 1 >= int(e->sigmas.size()))
        return false;
    *c = ErSdeCoef{};
    c->stage = std::min(3, i + 1);
    if (e->sigmas[i + 1] == 0) {
        c->last = true;
        return true;
    }
    // Three-stage update from the image estimates' first and second differences (er_sde.cpp:36-69); the
    // integrals of 1 / scaler over [lambda_t, lambda_s] are Riemann sums over 200 points.
    const double ls = e->lambdas[i], lt = e->lambdas[i + 1];
    const double alpha_s = e->sigmas[i] / ls, alpha_t = e->sigmas[i + 1] / lt;
    const double r = er_scaler(lt) / er_scaler(ls);
    c->c1 = alpha_t / alpha_s * r;
    c->c2 = alpha_t * (1 - r);
    const int points = 200;
    const double dt = lt - ls, h = -dt / points;
    double s = 0, su = 0;
    for (int k = 0; k < points; ++k) {
        const double pos = lt + k * h, sp = er_scaler(pos);
        s += 1 / sp;
        su += (pos - ls) / sp;
    }
    s *= h;
    su *= h;
    c->c3 = alpha_t * (dt + s * er_scaler(lt));
    c->c4 = alpha_t * (dt * dt / 2 + su * er_scaler(lt));
    c->d_den = c->stage >= 2 ? ls - e->lambdas[i - 1] : 1;
    c->u_den = c->stage >= 3 ? (ls - e->lambdas[i - 2]) / 2 : 1;
    c->cn = alpha_t * double(s_noise) * std::sqrt(std::max(0.0, lt * lt - ls * ls * r * r));
    return true;
}

double er_sde_sigma_d(const mkb_er_sde* e, int i)
{
    return e && i >= 0 && i < int(e->sigmas.size()) ? e->sigmas[i] : 0.0;
}

bool er_sde_dev_order(mkb_er_sde* e, int i)
{
    if (!e || (i != 0 && i != e->dev_next))
        return false;
    e->dev_next = i + 1;
    return true;
}

}  // namespace mkb
