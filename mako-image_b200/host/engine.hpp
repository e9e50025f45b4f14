// The reference's model / sampler API (src/image/engine.hpp) over the CUDA backend: a C++ mirror of image::Engine's
// denoising side and of QwenImage, so code written against the reference's Engine drives the B200 kernels.
//
// Kept from the reference, with the same names, argument meaning and error behaviour (std::runtime_error):
//   Engine::begin / step            (engine.hpp:165-166)   -> mkb_dit_begin / mkb_dit_step
//   Engine::sigmas / top_sigma      (engine.hpp:189-192)   -> mkb_sigmas / mkb_top_sigma
//   Engine::generate's loop         (engine.cpp:367-508)   -> Engine::denoise: CFG, Euler, ER-SDE
//   Engine::decode                  (engine.cpp:862-954)   -> Vae::decode (mkb_vae_decode)
//   Sdxl::begin / step              (sdxl.cpp:672-953)     -> Sdxl (mkb_unet_begin / mkb_unet_step)
//   Sampler, parse_sampler          (engine.hpp:49-53)
// Left out (outside the hot path): text encoding (prompt embeddings are an input); image I/O is in png.hpp.
#pragma once

#include "../../include/mkb_image.h"

#include <cstdint>
#include <functional>
#include <optional>
#include <span>
#include <stdexcept>
#include <string>
#include <string_view>
#include <vector>

namespace mkb::image {

enum class Sampler { euler, euler_ancestral, er_sde };
std::optional<Sampler> parse_sampler(std::string_view name);
const char* sampler_name(Sampler s);

// Throws std::runtime_error with the library's message for a failed call (the reference throws on bad shapes).
void check(mkb_status s, const char* what);

class Engine {
public:
    virtual ~Engine() = default;
    virtual const char* name() const = 0;
    virtual uint32_t default_steps() const = 0;
    virtual float default_guidance() const = 0;
    virtual bool predicts_noise() const { return false; }
    virtual Sampler default_sampler() const { return Sampler::euler; }
    // A token's latent values (Qwen-Image: 64, 16 channels x a 2x2 patch; SDXL: 16, 4 channels x 2x2).
    virtual uint32_t latent_width() const { return 64; }

    virtual void begin(std::span<const float> prompt, uint32_t h, uint32_t w, uint32_t slot = 0) = 0;
    virtual std::vector<float> step(std::span<const float> latents, float sigma, uint32_t slot = 0) = 0;

    virtual std::vector<float> sigmas(uint32_t steps, uint32_t tokens,
                                      std::optional<float> terminal = std::nullopt) const;
    virtual float top_sigma(uint32_t tokens) const;

    // Engine::generate's denoising loop (engine.cpp:453-507) from prompt embeddings to the final latents: noise
    // from `noise` (or seeded; for a model that predicts the noise scaled to the top level's sqrt(1 + sigma^2),
    // engine.cpp:453-458), guidance with the negative prompt's embeddings when given and scale != 1, then Euler,
    // Euler ancestral or ER-SDE steps. Decoding is the VAE's (Vae::decode).
    struct Request {
        std::span<const float> prompt, negative;  // the model's begin() layout; negative empty: no guidance
        uint32_t h = 64, w = 64;                   // latent grid (tokens)
        uint32_t steps = 0;                        // 0: default_steps()
        std::optional<float> guidance, terminal;
        std::optional<Sampler> sampler;
        std::span<const float> noise;              // [h * w][latent_width()]; empty: from seed
        uint64_t seed = 0;
        std::function<void(uint32_t, uint32_t)> progress;
    };
    std::vector<float> denoise(const Request& r);

protected:
    mkb_schedule sched_{};
    // A batched guided step when the backend has one (both slots in one pass); false: run two step() calls.
    virtual bool guided_step(std::vector<float>& x, float sigma, float sigma_next, float scale)
    {
        (void)x, (void)sigma, (void)sigma_next, (void)scale;
        return false;
    }
};

// Qwen-Image-style MMDiT on the B200 kernels (mkb_dit). `variant` picks the reference's own block math
// (MKB_VARIANT_REF21) or the Qwen-Image(-1) shape (MKB_VARIANT_QWEN1).
class QwenImage final : public Engine {
public:
    explicit QwenImage(const mkb_dit_config& cfg);
    ~QwenImage() override;
    QwenImage(const QwenImage&) = delete;
    QwenImage& operator=(const QwenImage&) = delete;

    const char* name() const override { return "Qwen-Image (B200)"; }
    uint32_t default_steps() const override { return 40; }
    float default_guidance() const override { return 4.0f; }

    void begin(std::span<const float> prompt, uint32_t h, uint32_t w, uint32_t slot = 0) override;
    std::vector<float> step(std::span<const float> latents, float sigma, uint32_t slot = 0) override;

    // Engine::denoise with the latents kept on the device: the guided velocity of both slots in one pass
    // (mkb_dit_guided_velocity_dev) and the sampler update on the device (mkb_axpy_dev / mkb_euler_ancestral_dev /
    // mkb_er_sde_step_dev) on one stream, so only the final latents come back. Same initial latents as denoise();
    // the ancestral and ER-SDE noise is the device's counter-based stream keyed by the seed.
    std::vector<float> denoise_device(const Request& r);

    // Synthetic weights by seed (mkb_dit_init_random), or named weights from host memory (mkb_dit_weight_write).
    void init_random(uint64_t seed, float std = 0.02f);
    void load_weight(const std::string& name, std::span<const float> values);
    mkb_dit* handle() { return d_; }

protected:
    bool guided_step(std::vector<float>& x, float sigma, float sigma_next, float scale) override;

private:
    mkb_dit* d_ = nullptr;
    mkb_dit_config cfg_{};
    uint32_t gh_ = 0, gw_ = 0;
    uint32_t prompt_rows_[2] = {0, 0};
};

// The SDXL UNet on the B200 kernels (mkb_unet): an eps-predicting model with the discrete SDXL schedule.
class Sdxl final : public Engine {
public:
    explicit Sdxl(const mkb_unet_config& cfg);
    ~Sdxl() override;
    Sdxl(const Sdxl&) = delete;
    Sdxl& operator=(const Sdxl&) = delete;

    const char* name() const override { return "SDXL (B200)"; }
    uint32_t default_steps() const override { return 28; }
    float default_guidance() const override { return 6.0f; }
    bool predicts_noise() const override { return true; }
    uint32_t latent_width() const override { return 16; }

    // prompt: [S, then S x context_dim context rows, then pooled_dim pooled values], the reference's prompt
    // embeddings layout (Sdxl::begin, sdxl.cpp:672-681).
    void begin(std::span<const float> prompt, uint32_t h, uint32_t w, uint32_t slot = 0) override;
    std::vector<float> step(std::span<const float> latents, float sigma, uint32_t slot = 0) override;
    std::vector<float> sigmas(uint32_t steps, uint32_t tokens,
                              std::optional<float> terminal = std::nullopt) const override;
    float top_sigma(uint32_t tokens) const override;

    void init_random(uint64_t seed, float std = 0.02f);
    mkb_unet* handle() { return u_; }

protected:
    bool guided_step(std::vector<float>& x, float sigma, float sigma_next, float scale) override;

private:
    mkb_unet* u_ = nullptr;
    mkb_unet_config cfg_{};
    uint32_t gh_ = 0, gw_ = 0;
    uint32_t ctx_rows_[2] = {0, 0};
};

// The VAE decoder (mkb_vae): Engine::decode's tokens-to-image pass.
class Vae {
public:
    explicit Vae(const mkb_vae_config& cfg);
    ~Vae();
    Vae(const Vae&) = delete;
    Vae& operator=(const Vae&) = delete;

    // latents [h * w][4 * latent] to RGBA [16 h][16 w][4] in [-1, 1] (engine.cpp:862-954)
    std::vector<float> decode(std::span<const float> latents, uint32_t h, uint32_t w);
    // per token value: the decoder sees latents * std + mean (engine.cpp:890-898)
    void set_latent_stats(std::span<const float> mean, std::span<const float> std);
    void init_random(uint64_t seed, float std = 0.02f);
    // Weights from checkpoint files by their own names (mkb_vae_load_safetensors); returns the count written.
    int load(const std::vector<std::string>& files, bool strict = true);
    uint32_t latent_width() const { return uint32_t(4 * cfg_.latent); }
    mkb_vae* handle() { return v_; }

private:
    mkb_vae* v_ = nullptr;
    mkb_vae_config cfg_{};
};

}  // namespace mkb::image
