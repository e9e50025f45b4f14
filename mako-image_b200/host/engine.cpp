// The C++ Engine mirror over the C ABI (see engine.hpp).
#include "engine.hpp"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <random>

namespace mkb::image {

void check(mkb_status s, const char* what)
{
    if (s != MKB_OK)
        throw std::runtime_error(std::string(what) + ": " + mkb_last_error());
}

std::optional<Sampler> parse_sampler(std::string_view n)
{
    if (n == "euler")
        return Sampler::euler;
    if (n == "euler_a" || n == "euler_ancestral")
        return Sampler::euler_ancestral;
    if (n == "er_sde")
        return Sampler::er_sde;
    return std::nullopt;
}

const char* sampler_name(Sampler s)
{
    switch (s) {
    case Sampler::euler: return "euler";
    case Sampler::euler_ancestral: return "euler_a";
    case Sampler::er_sde: return "er_sde";
    }
    return "";
}

std::vector<float> Engine::sigmas(uint32_t steps, uint32_t tokens, std::optional<float> terminal) const
{
    mkb_schedule s = sched_;
    if (s.max_seq == 0)
        mkb_schedule_default(&s);
    if (terminal)
        s.terminal = *terminal;
    std::vector<float> out(steps + 1);
    check(mkb_sigmas(&s, steps, tokens, out.data()), "sigmas");
    return out;
}

float Engine::top_sigma(uint32_t tokens) const
{
    mkb_schedule s = sched_;
    if (s.max_seq == 0)
        mkb_schedule_default(&s);
    return mkb_top_sigma(&s, tokens);
}

std::vector<float> Engine::denoise(const Request& r)
{
    const uint32_t N = r.h * r.w, lat = latent_width();
    const Sampler sampler = r.sampler.value_or(default_sampler());
    if (sampler == Sampler::euler_ancestral && !predicts_noise())
        throw std::runtime_error(std::string(name()) + ": Euler a needs a model that predicts the noise");
    std::vector<float> x(size_t(N) * lat);
    std::mt19937_64 rng(r.seed);
    std::normal_distribution<float> nd;
    if (!r.noise.empty()) {
        if (r.noise.size() != x.size())
            throw std::runtime_error("noise must be [h * w][" + std::to_string(latent_width()) + "]");
        std::copy(r.noise.begin(), r.noise.end(), x.begin());
    } else {
        for (float& v : x)
            v = nd(rng);
    }
    const auto sig = sigmas(r.steps ? r.steps : default_steps(), N, r.terminal);
    const uint32_t steps = uint32_t(sig.size() - 1);
    // A model that predicts the noise starts from noise at the top level's scale, sqrt(1 + sigma^2).
    if (predicts_noise()) {
        const float s0 = std::sqrt(1.0f + sig[0] * sig[0]);
        for (float& v : x)
            v *= s0;
    }
    begin(r.prompt, r.h, r.w, 0);
    const float scale = r.guidance.value_or(default_guidance());
    const bool guided = scale != 1.0f && !r.negative.empty();
    if (guided)
        begin(r.negative, r.h, r.w, 1);
    mkb_er_sde* er = nullptr;
    std::vector<float> noise;
    if (sampler == Sampler::er_sde) {
        check(mkb_er_sde_create(sig.data(), int(sig.size()), predicts_noise() ? 0 : 1, top_sigma(N), &er), "ER-SDE");
        noise.resize(x.size());
    }
    struct Guard {
        mkb_er_sde* e;
        ~Guard() { mkb_er_sde_destroy(e); }
    } guard{er};
    for (uint32_t i = 0; i < steps; ++i) {
        const float s = er ? mkb_er_sde_sigma(er, int(i)) : sig[i];
        // Plain guided Euler runs as one batched device pass (cond + uncond, update fused).
        if (!er && sampler == Sampler::euler && guided && guided_step(x, s, sig[i + 1], scale)) {
            if (r.progress)
                r.progress(i + 1, steps);
            continue;
        }
        auto v = step(x, s, 0);
        if (guided) {
            const auto neg = step(x, s, 1);
            for (size_t j = 0; j < v.size(); ++j)
                v[j] = neg[j] + scale * (v[j] - neg[j]);
        }
        if (er) {
            for (size_t j = 0; j < v.size(); ++j)
                v[j] = x[j] - s * v[j];
            if (sig[i + 1] > 0)
                for (float& n : noise)
                    n = nd(rng);
            check(mkb_er_sde_step(er, int(i), x.data(), v.data(), noise.data(), long(x.size()), 1.0f), "ER-SDE step");
        } else if (sampler == Sampler::euler_ancestral) {
            const double from = sig[i], to = sig[i + 1];
            const double up = std::min(to, std::sqrt(to * to * (from * from - to * to) / (from * from)));
            const float dt = float(std::sqrt(to * to - up * up) - from);
            for (size_t j = 0; j < x.size(); ++j)
                x[j] += dt * v[j];
            if (up > 0)
                for (float& xv : x)
                    xv += float(up) * nd(rng);
        } else {
            mkb_guided_euler(x.data(), v.data(), nullptr, 1.0f, sig[i], sig[i + 1], long(x.size()));
        }
        if (r.progress)
            r.progress(i + 1, steps);
    }
    return x;
}

QwenImage::QwenImage(const mkb_dit_config& cfg) : cfg_(cfg)
{
    mkb_schedule_default(&sched_);
    check(mkb_dit_create(&cfg, &d_), "create");
}

QwenImage::~QwenImage() { mkb_dit_destroy(d_); }

void QwenImage::init_random(uint64_t seed, float std) { check(mkb_dit_init_random(d_, seed, std), "init_random"); }

void QwenImage::load_weight(const std::string& name, std::span<const float> values)
{
    check(mkb_dit_weight_write(d_, name.c_str(), values.data()), "load_weight");
}

void QwenImage::begin(std::span<const float> prompt, uint32_t h, uint32_t w, uint32_t slot)
{
    const uint32_t td = uint32_t(cfg_.text_dim);
    if (prompt.empty() || prompt.size() % td)
        throw std::runtime_error("prompt embeddings must be rows of " + std::to_string(td));
    check(mkb_dit_begin(d_, prompt.data(), int(prompt.size() / td), int(h), int(w), int(slot)), "begin");
    gh_ = h;
    gw_ = w;
    if (slot < 2)
        prompt_rows_[slot] = uint32_t(prompt.size() / td);
}

std::vector<float> QwenImage::step(std::span<const float> latents, float sigma, uint32_t slot)
{
    const uint64_t N = uint64_t(gh_) * gw_;
    if (latents.size() != N * latent_width())
        throw std::runtime_error("latents must be [h * w][64]");
    std::vector<float> out(latents.size());
    check(mkb_dit_step(d_, latents.data(), sigma, out.data(), int(slot)), "step");
    return out;
}

std::vector<float> QwenImage::denoise_device(const Request& r)
{
    const uint32_t N = r.h * r.w;
    const long n = long(N) * latent_width();
    const Sampler sampler = r.sampler.value_or(default_sampler());
    if (sampler == Sampler::euler_ancestral && !predicts_noise())
        throw std::runtime_error(std::string(name()) + ": Euler a needs a model that predicts the noise");
    std::vector<float> x(static_cast<size_t>(n));
    std::mt19937_64 rng(r.seed);
    std::normal_distribution<float> nd;
    if (!r.noise.empty()) {
        if (r.noise.size() != x.size())
            throw std::runtime_error("noise must be [h * w][" + std::to_string(latent_width()) + "]");
        std::copy(r.noise.begin(), r.noise.end(), x.begin());
    } else {
        for (float& v : x)
            v = nd(rng);
    }
    const auto sig = sigmas(r.steps ? r.steps : default_steps(), N, r.terminal);
    const uint32_t steps = uint32_t(sig.size() - 1);
    begin(r.prompt, r.h, r.w, 0);
    const float scale = r.guidance.value_or(default_guidance());
    const bool guided = scale != 1.0f && !r.negative.empty();
    if (guided)
        begin(r.negative, r.h, r.w, 1);
    const bool batched = guided && prompt_rows_[0] == prompt_rows_[1] && cfg_.max_batch >= 2 && cfg_.slots >= 2;

    // One stream for the model's and the sampler's launches; device buffers released on every exit path.
    struct Dev {
        cudaStream_t st = nullptr;
        float *x = nullptr, *v = nullptr, *u = nullptr, *state = nullptr;
        mkb_er_sde* er = nullptr;
        ~Dev()
        {
            if (st)
                cudaStreamSynchronize(st);
            for (float* p : {x, v, u, state})
                if (p)
                    cudaFree(p);
            if (st)
                cudaStreamDestroy(st);
            mkb_er_sde_destroy(er);
        }
    } dev;
    auto cu = [](cudaError_t e, const char* what) {
        if (e != cudaSuccess)
            throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
    };
    cu(cudaStreamCreateWithFlags(&dev.st, cudaStreamNonBlocking), "stream");
    cu(cudaMalloc(&dev.x, size_t(n) * 4), "latents");
    cu(cudaMalloc(&dev.v, size_t(n) * 4), "velocity");
    if (guided && !batched)
        cu(cudaMalloc(&dev.u, size_t(n) * 4), "velocity");
    if (sampler == Sampler::er_sde) {
        check(mkb_er_sde_create(sig.data(), int(sig.size()), predicts_noise() ? 0 : 1, top_sigma(N), &dev.er),
              "ER-SDE");
        cu(cudaMalloc(&dev.state, size_t(2 * n) * 4), "ER-SDE state");
    }
    cu(cudaMemcpyAsync(dev.x, x.data(), size_t(n) * 4, cudaMemcpyHostToDevice, dev.st), "latents upload");
    // The noise stream's key from the seed (a splitmix64 step of it).
    uint64_t key = r.seed + 0x9E3779B97F4A7C15ull;
    key = (key ^ (key >> 30)) * 0xBF58476D1CE4E5B9ull;
    key = (key ^ (key >> 27)) * 0x94D049BB133111EBull;
    key ^= key >> 31;
    const int slot0 = 0, slot1 = 1;
    for (uint32_t i = 0; i < steps; ++i) {
        const float s = dev.er ? mkb_er_sde_sigma(dev.er, int(i)) : sig[i];
        if (batched) {
            check(mkb_dit_guided_velocity_dev(d_, 1, dev.x, s, scale, dev.v, dev.st), "guided velocity");
        } else {
            check(mkb_dit_step_batch_dev(d_, 1, &slot0, dev.x, &s, dev.v, dev.st), "step");
            if (guided) {
                check(mkb_dit_step_batch_dev(d_, 1, &slot1, dev.x, &s, dev.u, dev.st), "step");
                check(mkb_cfg_combine_dev(dev.v, dev.v, dev.u, scale, n, dev.st), "guidance");
            }
        }
        const uint64_t off = uint64_t(i) * uint64_t(n);
        if (dev.er)
            check(mkb_er_sde_step_dev(dev.er, int(i), dev.x, dev.v, dev.state, key, off, n, 1.0f, dev.st), "ER-SDE");
        else if (sampler == Sampler::euler_ancestral)
            check(mkb_euler_ancestral_dev(dev.x, dev.v, sig[i], sig[i + 1], key, off, n, dev.st), "Euler a");
        else
            check(mkb_axpy_dev(dev.x, dev.v, sig[i + 1] - sig[i], n, dev.st), "Euler");
        if (r.progress)
            r.progress(i + 1, steps);
    }
    cu(cudaMemcpyAsync(x.data(), dev.x, size_t(n) * 4, cudaMemcpyDeviceToHost, dev.st), "latents download");
    cu(cudaStreamSynchronize(dev.st), "denoise");
    uint32_t bits = 0;
    check(mkb_check_kernels(&bits), "kernel status");
    if (bits)
        throw std::runtime_error("denoise_device: kernel status bits " + std::to_string(bits));
    return x;
}

bool QwenImage::guided_step(std::vector<float>& x, float sigma, float sigma_next, float scale)
{
    // Both slots batched needs equal prompt lengths (and, for the reference variant, equal step counts, which the
    // loop keeps).
    if (prompt_rows_[0] != prompt_rows_[1] || cfg_.max_batch < 2 || cfg_.slots < 2)
        return false;
    check(mkb_dit_step_cfg(d_, x.data(), sigma, sigma_next, scale), "guided step");
    return true;
}

// ------------------------------------------------------------------------------------------------ SDXL

Sdxl::Sdxl(const mkb_unet_config& cfg) : cfg_(cfg) { check(mkb_unet_create(&cfg, &u_), "create"); }

Sdxl::~Sdxl() { mkb_unet_destroy(u_); }

void Sdxl::init_random(uint64_t seed, float std) { check(mkb_unet_init_random(u_, seed, std), "init_random"); }

void Sdxl::begin(std::span<const float> prompt, uint32_t h, uint32_t w, uint32_t slot)
{
    if (slot > 1)
        throw std::runtime_error("slot must be 0 or 1");
    if (prompt.empty())
        throw std::runtime_error("prompt embeddings: no header");
    const uint32_t S = uint32_t(prompt[0]);
    if (!S || prompt.size() != 1 + uint64_t(S) * cfg_.context_dim + cfg_.pooled_dim)
        throw std::runtime_error("prompt embeddings: sizes do not add up");
    check(mkb_unet_begin(u_, prompt.data() + 1, int(S), prompt.data() + 1 + uint64_t(S) * cfg_.context_dim, int(h),
                         int(w), int(slot)),
          "begin");
    gh_ = h;
    gw_ = w;
    ctx_rows_[slot] = S;
}

std::vector<float> Sdxl::step(std::span<const float> latents, float sigma, uint32_t slot)
{
    if (latents.size() != uint64_t(gh_) * gw_ * latent_width())
        throw std::runtime_error("latents must be [h * w][16]");
    std::vector<float> out(latents.size());
    check(mkb_unet_step(u_, latents.data(), sigma, out.data(), int(slot)), "step");
    return out;
}

std::vector<float> Sdxl::sigmas(uint32_t steps, uint32_t tokens, std::optional<float> terminal) const
{
    (void)tokens, (void)terminal;  // the discrete schedule depends on neither
    std::vector<float> out(steps + 1);
    check(mkb_sdxl_sigmas(steps, out.data()), "sigmas");
    return out;
}

float Sdxl::top_sigma(uint32_t tokens) const { return sigmas(1, tokens)[0]; }

bool Sdxl::guided_step(std::vector<float>& x, float sigma, float sigma_next, float scale)
{
    if (ctx_rows_[0] != ctx_rows_[1] || cfg_.max_batch < 2 || cfg_.slots < 2)
        return false;
    // Both slots in one batched pass, then the guided Euler update on the host.
    const size_t n = x.size();
    std::vector<float> in(2 * n), out(2 * n);
    std::copy(x.begin(), x.end(), in.begin());
    std::copy(x.begin(), x.end(), in.begin() + long(n));
    const float s2[2] = {sigma, sigma};
    check(mkb_unet_step_batch(u_, 2, 0, in.data(), s2, out.data()), "guided step");
    mkb_guided_euler(x.data(), out.data(), out.data() + n, scale, sigma, sigma_next, long(n));
    return true;
}

// ------------------------------------------------------------------------------------------------ VAE

Vae::Vae(const mkb_vae_config& cfg) : cfg_(cfg) { check(mkb_vae_create(&cfg, &v_), "vae create"); }

Vae::~Vae() { mkb_vae_destroy(v_); }

std::vector<float> Vae::decode(std::span<const float> latents, uint32_t h, uint32_t w)
{
    if (latents.size() != uint64_t(h) * w * latent_width())
        throw std::runtime_error("latents must be [h * w][" + std::to_string(latent_width()) + "]");
    std::vector<float> img(uint64_t(16 * h) * (16 * w) * 4);
    check(mkb_vae_decode(v_, latents.data(), int(h), int(w), img.data()), "decode");
    return img;
}

void Vae::set_latent_stats(std::span<const float> mean, std::span<const float> std)
{
    if (mean.size() != std.size())
        throw std::runtime_error("latent statistics: as many means as deviations");
    check(mkb_vae_set_latent_stats(v_, mean.data(), std.data(), int(mean.size())), "latent statistics");
}

void Vae::init_random(uint64_t seed, float std) { check(mkb_vae_init_random(v_, seed, std), "vae init_random"); }

int Vae::load(const std::vector<std::string>& files, bool strict)
{
    std::vector<const char*> p;
    for (const auto& f : files)
        p.push_back(f.c_str());
    int n = 0;
    check(mkb_vae_load_safetensors(v_, p.data(), int(p.size()), strict ? 1 : 0, &n), "vae load");
    return n;
}

}  // namespace mkb::image
