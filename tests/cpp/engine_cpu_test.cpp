// The C++ Engine mirror's denoising loop over a made-up model (the reference's own testing pattern,
// tests/er_sde_test.cpp:13-28): no GPU. Checks the schedule, the guided Euler loop against a hand-rolled loop, and
// ER-SDE through Engine::denoise against mkb_er_sde driven directly. Exit 0 on success.
#include "../../mako-image_b200/host/engine.hpp"

#include <cmath>
#include <cstdio>
#include <random>
#include <vector>

namespace {

int failures = 0;

void expect(bool ok, const char* what)
{
    std::printf("  %-4s %s\n", ok ? "ok" : "FAIL", what);
    failures += !ok;
}

// v = tanh(x (0.6 + 0.2 sigma)) + 0.1 cos(j + 3 sigma) for the prompt slot, a scaled copy for the negative one.
class Fake final : public mkb::image::Engine {
public:
    const char* name() const override { return "fake"; }
    uint32_t default_steps() const override { return 6; }
    float default_guidance() const override { return 3.0f; }
    void begin(std::span<const float>, uint32_t h, uint32_t w, uint32_t) override { n_ = h * w * 64; }
    std::vector<float> step(std::span<const float> x, float s, uint32_t slot) override
    {
        std::vector<float> v(x.size());
        for (size_t j = 0; j < x.size(); ++j)
            v[j] = std::tanh(x[j] * (0.6f + 0.2f * s)) + 0.1f * std::cos(float(j % 64) + 3 * s) * (slot ? 0.5f : 1.0f);
        return v;
    }
    uint32_t n_ = 0;
};

}  // namespace

int main()
{
    Fake m;
    const std::vector<float> prompt(4), neg(4);
    std::vector<float> noise(2 * 2 * 64);
    for (size_t j = 0; j < noise.size(); ++j)
        noise[j] = std::sin(0.37f * float(j));
    // Schedule: decreasing from 1 to 0, first 1, last before 0 at t = 1/steps.
    const auto sig = m.sigmas(6, 4);
    expect(sig.size() == 7 && sig[0] == 1.0f && sig[6] == 0.0f, "sigmas: 6 levels then 0");
    bool dec = true;
    for (size_t i = 0; i + 1 < sig.size(); ++i)
        dec &= sig[i] > sig[i + 1];
    expect(dec, "sigmas decrease");

    // Guided Euler through denoise() against the loop written out.
    mkb::image::Engine::Request r;
    r.prompt = prompt;
    r.negative = neg;
    r.h = 2;
    r.w = 2;
    r.noise = noise;
    const auto got = m.denoise(r);
    std::vector<float> x(noise);
    for (size_t i = 0; i + 1 < sig.size(); ++i) {
        auto v = m.step(x, sig[i], 0);
        const auto u = m.step(x, sig[i], 1);
        for (size_t j = 0; j < x.size(); ++j)
            x[j] += (sig[i + 1] - sig[i]) * (u[j] + 3.0f * (v[j] - u[j]));
    }
    double err = 0;
    for (size_t j = 0; j < x.size(); ++j)
        err = std::max(err, double(std::fabs(x[j] - got[j])));
    expect(err < 1e-6, "guided Euler loop");

    // ER-SDE through denoise() (flow model, no guidance) against mkb_er_sde driven directly with the same noise.
    r.negative = {};
    r.sampler = mkb::image::Sampler::er_sde;
    r.seed = 7;
    const auto er_got = m.denoise(r);
    mkb_er_sde* er = nullptr;
    mkb::image::check(mkb_er_sde_create(sig.data(), int(sig.size()), 1, m.top_sigma(4), &er), "er");
    std::vector<float> y(noise), z(noise.size());
    std::mt19937_64 rng(7);
    std::normal_distribution<float> nd;
    for (size_t j = 0; j < noise.size(); ++j)  // denoise() draws its start noise only without r.noise; none here
        (void)j;
    for (size_t i = 0; i + 1 < sig.size(); ++i) {
        const float s = mkb_er_sde_sigma(er, int(i));
        auto v = m.step(y, s, 0);
        for (size_t j = 0; j < y.size(); ++j)
            v[j] = y[j] - s * v[j];
        if (sig[i + 1] > 0)
            for (float& n : z)
                n = nd(rng);
        mkb::image::check(mkb_er_sde_step(er, int(i), y.data(), v.data(), z.data(), long(y.size()), 1.0f), "step");
    }
    mkb_er_sde_destroy(er);
    err = 0;
    for (size_t j = 0; j < y.size(); ++j)
        err = std::max(err, double(std::fabs(y[j] - er_got[j])));
    expect(err < 1e-6, "ER-SDE loop");

    // Errors surface as std::runtime_error, as in the reference.
    bool threw = false;
    try {
        r.sampler = mkb::image::Sampler::euler_ancestral;
        m.denoise(r);
    } catch (const std::runtime_error&) {
        threw = true;
    }
    expect(threw, "Euler a refused for a velocity model");
    std::printf("%s\n", failures ? "FAILED" : "passed");
    return failures ? 1 : 0;
}
