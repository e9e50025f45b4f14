// The C++ Engine mirror on the B200 kernels: a small Qwen-Image-shape model (random weights), three guided Euler
// steps through Engine::denoise (cond + uncond batched on the device, update fused) against the same steps as two
// step() calls combined on the host, for both block variants; then the device loop (QwenImage::denoise_device)
// against the host loop, and its ER-SDE run for reproducibility. Then the SDXL side through the C ABI: Sdxl::denoise
// (noise at the top level's scale, cond + uncond batched) against unbatched step() calls, and Vae::decode of its
// latents (mkb_vae_decode). Exit 0 on success.
#include "../../mako-image_b200/host/engine.hpp"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <stdexcept>
#include <vector>

int main()
{
    int failures = 0;
    for (int variant : {MKB_VARIANT_QWEN1, MKB_VARIANT_REF21}) {
        mkb_dit_config c{};
        c.variant = variant;
        c.hidden = 512;
        c.heads = 4;
        c.ffn = 1024;
        c.blocks = 2;
        c.text_dim = 256;
        c.max_batch = 2;
        c.max_text_tokens = 32;
        c.max_image_tokens = 64;
        c.slots = 2;
        const uint32_t h = 8, w = 8, S = 24, N = h * w;
        std::vector<float> prompt(S * 256), neg(S * 256), noise(N * 64);
        for (size_t j = 0; j < prompt.size(); ++j) {
            prompt[j] = std::sin(0.1f * float(j));
            neg[j] = std::cos(0.07f * float(j));
        }
        for (size_t j = 0; j < noise.size(); ++j)
            noise[j] = std::sin(0.37f * float(j) + 1.0f);
        mkb::image::QwenImage a(c), b(c);
        a.init_random(11);
        b.init_random(11);
        mkb::image::Engine::Request r;
        r.prompt = prompt;
        r.negative = neg;
        r.h = h;
        r.w = w;
        r.steps = 3;
        r.noise = noise;
        const auto got = a.denoise(r);
        // The same three steps, unbatched.
        const auto sig = b.sigmas(3, N);
        b.begin(prompt, h, w, 0);
        b.begin(neg, h, w, 1);
        std::vector<float> x(noise);
        for (int i = 0; i < 3; ++i) {
            const auto v = b.step(x, sig[i], 0);
            const auto u = b.step(x, sig[i], 1);
            mkb_guided_euler(x.data(), v.data(), u.data(), 4.0f, sig[i], sig[i + 1], long(x.size()));
        }
        double err = 0, mx = 0;
        bool finite = true;
        for (size_t j = 0; j < x.size(); ++j) {
            err = std::max(err, double(std::fabs(x[j] - got[j])));
            mx = std::max(mx, double(std::fabs(x[j])));
            finite &= std::isfinite(got[j]);
        }
        const bool ok = finite && err <= 1e-4 * std::max(1.0, mx);
        std::printf("  %-4s variant %d: batched guided steps vs two step() calls, max-abs %.3e\n", ok ? "ok" : "FAIL",
                    variant, err);
        failures += !ok;

        // The device loop (latents stay on the GPU): guided Euler equals the host loop's result.
        mkb::image::QwenImage e(c);
        e.init_random(11);
        const auto dev = e.denoise_device(r);
        double derr = 0;
        for (size_t j = 0; j < dev.size(); ++j)
            derr = std::max(derr, double(std::fabs(dev[j] - got[j])));
        const bool dok = derr <= 1e-4 * std::max(1.0, mx);
        std::printf("  %-4s variant %d: device loop (guided Euler) vs host loop, max-abs %.3e\n", dok ? "ok" : "FAIL",
                    variant, derr);
        failures += !dok;

        // Device ER-SDE: finite, reproducible from the seed, and not the Euler result.
        mkb::image::Engine::Request r2 = r;
        r2.sampler = mkb::image::Sampler::er_sde;
        r2.seed = 5;
        mkb::image::QwenImage f(c), g(c);
        f.init_random(11);
        g.init_random(11);
        const auto e1 = f.denoise_device(r2), e2 = g.denoise_device(r2);
        bool same = e1 == e2, fin = true;
        double diff = 0;
        for (size_t j = 0; j < e1.size(); ++j) {
            fin &= std::isfinite(e1[j]);
            diff = std::max(diff, double(std::fabs(e1[j] - dev[j])));
        }
        const bool eok = same && fin && diff > 0;
        std::printf("  %-4s variant %d: device ER-SDE reproducible (%d), finite (%d), differs from Euler by %.3e\n",
                    eok ? "ok" : "FAIL", variant, int(same), int(fin), diff);
        failures += !eok;
    }
    {
        // SDXL: a reduced UNet (the full model's block structure) and VAE.
        mkb_unet_config c{};
        const int ch[3] = {64, 128, 256}, dep[3] = {0, 1, 1};
        for (int k = 0; k < 3; ++k) {
            c.channels[k] = ch[k];
            c.depth[k] = dep[k];
        }
        c.layers = 2;
        c.context_dim = 256;
        c.pooled_dim = 128;
        c.max_batch = 2;
        c.max_gh = 8;
        c.max_gw = 16;
        c.max_context = 77;
        c.slots = 2;
        const uint32_t h = 8, w = 16, S = 20, N = h * w;
        // The reference's prompt layout: [S, S x context_dim, pooled_dim].
        auto embeds = [&](float f) {
            std::vector<float> p = {float(S)};
            for (uint32_t j = 0; j < S * 256 + 128; ++j)
                p.push_back(std::sin(f * float(j) + 0.3f));
            return p;
        };
        const auto prompt = embeds(0.11f), neg = embeds(0.05f);
        std::vector<float> noise(N * 16);
        for (size_t j = 0; j < noise.size(); ++j)
            noise[j] = std::sin(0.41f * float(j) + 2.0f);
        mkb::image::Sdxl a(c), b(c);
        a.init_random(7);
        b.init_random(7);
        mkb::image::Engine::Request r;
        r.prompt = prompt;
        r.negative = neg;
        r.h = h;
        r.w = w;
        r.steps = 3;
        r.guidance = 5.0f;
        r.noise = noise;
        const auto got = a.denoise(r);
        const auto sig = b.sigmas(3, N);
        b.begin(prompt, h, w, 0);
        b.begin(neg, h, w, 1);
        std::vector<float> x(noise);
        const float s0 = std::sqrt(1.0f + sig[0] * sig[0]);
        for (float& v : x)
            v *= s0;
        for (int i = 0; i < 3; ++i) {
            const auto v = b.step(x, sig[i], 0);
            const auto u = b.step(x, sig[i], 1);
            mkb_guided_euler(x.data(), v.data(), u.data(), 5.0f, sig[i], sig[i + 1], long(x.size()));
        }
        double err = 0, mx = 0;
        bool finite = true;
        for (size_t j = 0; j < x.size(); ++j) {
            err = std::max(err, double(std::fabs(x[j] - got[j])));
            mx = std::max(mx, double(std::fabs(x[j])));
            finite &= std::isfinite(got[j]);
        }
        const bool ok = finite && err <= 1e-4 * std::max(1.0, mx);
        std::printf("  %-4s sdxl: batched guided steps vs two step() calls, max-abs %.3e\n", ok ? "ok" : "FAIL", err);
        failures += !ok;

        mkb_vae_config vc{};
        const int vch[4] = {128, 128, 128, 256};
        for (int k = 0; k < 4; ++k)
            vc.channels[k] = vch[k];
        vc.layers = 1;
        vc.latent = 4;
        vc.scale = 0.13025f;
        vc.max_gh = int(h);
        vc.max_gw = int(w);
        mkb::image::Vae vae(vc);
        vae.init_random(9);
        const auto img = vae.decode(got, h, w);
        bool vok = img.size() == size_t(16 * h) * (16 * w) * 4;
        for (size_t j = 0; vok && j < img.size(); ++j)
            vok = std::isfinite(img[j]) && img[j] >= -1.0f && img[j] <= 1.0f && (j % 4 != 3 || img[j] == 1.0f);
        bool threw = false;
        try {
            vae.decode(std::vector<float>(7), h, w);
        } catch (const std::runtime_error&) {
            threw = true;
        }
        vok = vok && threw;
        std::printf("  %-4s sdxl: VAE decode to RGBA in [-1, 1], wrong latent size rejected\n", vok ? "ok" : "FAIL");
        failures += !vok;
    }
    std::printf("%s\n", failures ? "FAILED" : "passed");
    return failures ? 1 : 0;
}
