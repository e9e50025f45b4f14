// mako_image: prompt embeddings in, PNG out, on the B200 kernels. The counterpart of the reference's driver
// (tools/mako_image.cpp:68-277): open a model, run Engine::generate's denoising loop, decode with the VAE, convert to
// 8-bit and write a PNG with its provenance chunks. Text encoding is not part of this library, so the prompt's
// embeddings come from a safetensors file (or, without one, seeded synthetic embeddings); the positional prompt is
// recorded in the PNG as the reference records it.
//
//   mako_image [options] <model dir | random> <prompt>
//
// Models: --model qwen (the Qwen-Image-style MMDiT, mkb_dit, denoised with the latents on the device, decoded by a
// 16-channel AutoencoderKL decoder) or --model sdxl (the SDXL UNet, mkb_unet, and the SDXL VAE). A model directory
// holds transformer/ (or unet/) and vae/ safetensors files, loaded by their checkpoint tensor names; "random" makes
// seeded random weights of the shapes the options give (for tests and timing).
#include "../host/engine.hpp"
#include "../host/png.hpp"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <filesystem>
#include <map>
#include <memory>
#include <random>
#include <sstream>
#include <string>
#include <vector>

namespace fs = std::filesystem;
using mkb::image::check;

namespace {

std::vector<int> int_list(const std::string& s)
{
    std::vector<int> v;
    std::stringstream ss(s);
    std::string t;
    while (std::getline(ss, t, ','))
        v.push_back(std::stoi(t));
    return v;
}

// Every tensor of a safetensors file as fp32 (the library's reader).
std::map<std::string, std::vector<float>> read_tensors(const std::string& path)
{
    mkb_st_file* f = nullptr;
    check(mkb_st_open(path.c_str(), &f), path.c_str());
    std::map<std::string, std::vector<float>> out;
    for (int i = 0; i < mkb_st_count(f); ++i) {
        const char *name = nullptr, *dtype = nullptr;
        int64_t dims[8];
        int nd = 0;
        check(mkb_st_info(f, i, &name, &dtype, dims, &nd), "safetensors info");
        int64_t count = 1;
        for (int k = 0; k < nd; ++k)
            count *= dims[k];
        std::vector<float> values(static_cast<size_t>(count));
        if (mkb_st_read_f32(f, name, values.data(), count) == MKB_OK)
            out[name] = std::move(values);
    }
    mkb_st_close(f);
    return out;
}

// The *.safetensors files of a model part: <dir>/<part>/, or <dir>/<part> itself when it is a file.
std::vector<std::string> part_files(const fs::path& dir, std::initializer_list<const char*> parts)
{
    std::vector<std::string> files;
    for (const char* part : parts) {
        const fs::path p = dir / part;
        if (fs::is_regular_file(p))
            return {p.string()};
        if (fs::is_directory(p)) {
            for (const auto& e : fs::directory_iterator(p))
                if (e.path().extension() == ".safetensors")
                    files.push_back(e.path().string());
            if (!files.empty())
                break;
        }
    }
    std::sort(files.begin(), files.end());
    if (files.empty())
        throw std::runtime_error("no safetensors files under " + dir.string() + " for this model part");
    return files;
}

std::vector<float> seeded_normals(size_t n, uint64_t seed)
{
    std::mt19937_64 r(seed);
    std::normal_distribution<float> nd;
    std::vector<float> v(n);
    for (float& x : v)
        x = nd(r);
    return v;
}

struct Options {
    std::string model = "qwen", variant = "qwen1", out = "image.png", embeds, lora, latents_out, latent_stats;
    std::vector<int> dims = {3072, 24, 12288, 60, 3584};
    std::vector<int> unet_ch = {320, 640, 1280}, unet_depth = {0, 2, 10}, vae_ch = {128, 256, 512, 512};
    int vae_layers = 2;
    uint32_t width = 1024, height = 1024, steps = 0, count = 1;
    uint64_t seed = 0, weights_seed = 1;
    std::optional<float> guidance;
    std::optional<mkb::image::Sampler> sampler;
    float lora_scale = 1.0f;
    bool rgb = false;
};

const char* kUsage =
    "usage: mako_image [options] <model dir | random> <prompt>\n"
    "  -o FILE               the PNG to write (default image.png; image-N.png after the first of --count)\n"
    "  --model qwen|sdxl     the denoiser (default qwen)\n"
    "  --variant qwen1|ref21 the Qwen-style block math (default qwen1)\n"
    "  --dims D,H,F,B,T      qwen: hidden, heads, FFN, blocks, text width (default 3072,24,12288,60,3584)\n"
    "  --unet-channels A,B,C / --unet-depth A,B,C   sdxl UNet widths and transformer depths\n"
    "  --vae-channels A,B,C,D / --vae-layers N      VAE decoder widths (output side first) and layers\n"
    "  --embeds FILE         prompt embeddings (.safetensors). qwen: prompt [S][T] (+ negative); sdxl: context\n"
    "                        [S][2048], pooled [1280] (+ negative_context, negative_pooled). Default: seeded\n"
    "  --latent-stats FILE   the VAE's latent statistics (.safetensors: mean, std per latent channel)\n"
    "  --width N --height N  pixels, multiples of 16 (sdxl: width a multiple of 256) (default 1024)\n"
    "  --steps N --seed N --count N --guidance F --sampler euler|euler_a|er_sde --rgb\n"
    "  --lora FILE[:SCALE]   merge a LoRA into the denoiser\n"
    "  --weights-seed N      seed of the random weights of model \"random\" (default 1)\n"
    "  --latents-out FILE    also write the first image's final latents (raw fp32, [h/16 * w/16][token values])\n";

}  // namespace

int main(int argc, char** argv)
{
    Options o;
    std::vector<std::string> pos;
    try {
        for (int i = 1; i < argc; ++i) {
            const std::string a = argv[i];
            auto val = [&]() -> std::string {
                if (i + 1 >= argc)
                    throw std::invalid_argument(a + " needs a value");
                return argv[++i];
            };
            if (a == "-o")
                o.out = val();
            else if (a == "--model")
                o.model = val();
            else if (a == "--variant")
                o.variant = val();
            else if (a == "--dims")
                o.dims = int_list(val());
            else if (a == "--unet-channels")
                o.unet_ch = int_list(val());
            else if (a == "--unet-depth")
                o.unet_depth = int_list(val());
            else if (a == "--vae-channels")
                o.vae_ch = int_list(val());
            else if (a == "--vae-layers")
                o.vae_layers = std::stoi(val());
            else if (a == "--embeds")
                o.embeds = val();
            else if (a == "--latent-stats")
                o.latent_stats = val();
            else if (a == "--width")
                o.width = uint32_t(std::stoul(val()));
            else if (a == "--height")
                o.height = uint32_t(std::stoul(val()));
            else if (a == "--steps")
                o.steps = uint32_t(std::stoul(val()));
            else if (a == "--seed")
                o.seed = std::stoull(val());
            else if (a == "--count")
                o.count = uint32_t(std::stoul(val()));
            else if (a == "--guidance")
                o.guidance = std::stof(val());
            else if (a == "--sampler") {
                o.sampler = mkb::image::parse_sampler(val());
                if (!o.sampler)
                    throw std::invalid_argument("--sampler: euler, euler_a or er_sde");
            } else if (a == "--rgb")
                o.rgb = true;
            else if (a == "--lora") {
                std::string v = val();
                const size_t c = v.rfind(':');
                if (c != std::string::npos && c > 0 && c + 1 < v.size() &&
                    v.find_first_not_of("0123456789.-", c + 1) == std::string::npos) {
                    o.lora_scale = std::stof(v.substr(c + 1));
                    v = v.substr(0, c);
                }
                o.lora = v;
            } else if (a == "--weights-seed")
                o.weights_seed = std::stoull(val());
            else if (a == "--latents-out")
                o.latents_out = val();
            else if (a == "-h" || a == "--help") {
                std::fputs(kUsage, stdout);
                return 0;
            } else if (!a.empty() && a[0] == '-')
                throw std::invalid_argument("unknown option " + a);
            else
                pos.push_back(a);
        }
        if (pos.size() != 2)
            throw std::invalid_argument("expected <model dir | random> <prompt>");
        if (o.width % 16 || o.height % 16 || !o.width || !o.height)
            throw std::invalid_argument("--width and --height: positive multiples of 16");
        if (o.model != "qwen" && o.model != "sdxl")
            throw std::invalid_argument("--model: qwen or sdxl");
        const bool random = pos[0] == "random";
        const uint32_t gh = o.height / 16, gw = o.width / 16;
        const bool qwen = o.model == "qwen";

        // The VAE decoder: 16 latent channels for the Qwen-style latents, 4 (SDXL, scale 0.13025) otherwise.
        if (o.vae_ch.size() != 4)
            throw std::invalid_argument("--vae-channels: four widths");
        mkb_vae_config vc{};
        for (int k = 0; k < 4; ++k)
            vc.channels[k] = o.vae_ch[k];
        vc.layers = o.vae_layers;
        vc.latent = qwen ? 16 : 4;
        vc.scale = qwen ? 1.0f : 0.13025f;
        vc.max_gh = int(gh);
        vc.max_gw = int(gw);
        mkb::image::Vae vae(vc);
        if (random)
            vae.init_random(o.weights_seed + 1);
        else
            vae.load(part_files(pos[0], {"vae"}));
        if (!o.latent_stats.empty()) {
            auto t = read_tensors(o.latent_stats);
            if (!t.count("mean") || !t.count("std") || t["mean"].size() != size_t(vc.latent) ||
                t["std"].size() != size_t(vc.latent))
                throw std::runtime_error("--latent-stats: mean and std, one per latent channel");
            std::vector<float> mean(4 * vc.latent), sd(4 * vc.latent);
            for (int i = 0; i < 4 * vc.latent; ++i) {  // token value i is channel i / 4's (a 2x2 patch)
                mean[i] = t["mean"][i / 4];
                sd[i] = t["std"][i / 4];
            }
            vae.set_latent_stats(mean, sd);
        }

        std::unique_ptr<mkb::image::Engine> engine;
        mkb::image::QwenImage* qimg = nullptr;
        std::vector<float> prompt, negative;
        if (qwen) {
            if (o.dims.size() != 5)
                throw std::invalid_argument("--dims: D,H,F,blocks,text width");
            mkb_dit_config c{};
            c.variant = o.variant == "ref21" ? MKB_VARIANT_REF21 : MKB_VARIANT_QWEN1;
            c.hidden = o.dims[0];
            c.heads = o.dims[1];
            c.ffn = o.dims[2];
            c.blocks = o.dims[3];
            c.text_dim = o.dims[4];
            c.max_batch = 2;
            c.max_image_tokens = int(gh * gw);
            c.slots = 2;
            std::map<std::string, std::vector<float>> emb;
            if (!o.embeds.empty()) {
                emb = read_tensors(o.embeds);
            } else {
                emb["prompt"] = seeded_normals(size_t(64) * c.text_dim, o.seed ^ 0x70726f6dull);
                emb["negative"] = seeded_normals(size_t(64) * c.text_dim, o.seed ^ 0x6e656761ull);
            }
            if (!emb.count("prompt") || emb["prompt"].size() % size_t(c.text_dim))
                throw std::runtime_error("embeddings: a prompt tensor of rows of the text width");
            prompt = emb["prompt"];
            if (emb.count("negative"))
                negative = emb["negative"];
            c.max_text_tokens = int(std::max(prompt.size(), negative.size()) / size_t(c.text_dim));
            auto q = std::make_unique<mkb::image::QwenImage>(c);
            if (random) {
                q->init_random(o.weights_seed);
            } else {
                const auto files = part_files(pos[0], {"transformer"});
                std::vector<const char*> p;
                for (const auto& f : files)
                    p.push_back(f.c_str());
                check(mkb_dit_load_safetensors(q->handle(), p.data(), int(p.size()), 1, nullptr), "transformer");
            }
            if (!o.lora.empty())
                check(mkb_dit_load_lora(q->handle(), o.lora.c_str(), o.lora_scale, nullptr), "lora");
            qimg = q.get();
            engine = std::move(q);
        } else {
            if (o.unet_ch.size() != 3 || o.unet_depth.size() != 3)
                throw std::invalid_argument("--unet-channels / --unet-depth: three values each");
            if (gw % 16)
                throw std::invalid_argument("sdxl: width a multiple of 256 pixels");
            mkb_unet_config c{};
            for (int k = 0; k < 3; ++k) {
                c.channels[k] = o.unet_ch[k];
                c.depth[k] = o.unet_depth[k];
            }
            c.layers = 2;
            c.context_dim = 2048;
            c.pooled_dim = 1280;
            c.max_batch = 2;
            c.max_gh = int(gh);
            c.max_gw = int(gw);
            c.max_context = 77;
            c.slots = 2;
            std::map<std::string, std::vector<float>> emb;
            if (!o.embeds.empty()) {
                emb = read_tensors(o.embeds);
            } else {
                emb["context"] = seeded_normals(size_t(77) * 2048, o.seed ^ 0x636f6e74ull);
                emb["pooled"] = seeded_normals(1280, o.seed ^ 0x706f6f6cull);
                emb["negative_context"] = seeded_normals(size_t(77) * 2048, o.seed ^ 0x6e636f6eull);
                emb["negative_pooled"] = seeded_normals(1280, o.seed ^ 0x6e706f6full);
            }
            // The reference's prompt layout: [S, context rows, pooled].
            auto pack = [&](const char* ctx, const char* pooled) {
                if (!emb.count(ctx) || !emb.count(pooled))
                    throw std::runtime_error(std::string("embeddings: ") + ctx + " and " + pooled + " needed");
                const auto& cv = emb.at(ctx);
                const auto& pv = emb.at(pooled);
                if (cv.empty() || cv.size() % 2048 || cv.size() / 2048 > 77 || pv.size() != 1280)
                    throw std::runtime_error("embeddings: context [S][2048] (S <= 77) and pooled [1280]");
                std::vector<float> p = {float(cv.size() / 2048)};
                p.insert(p.end(), cv.begin(), cv.end());
                p.insert(p.end(), pv.begin(), pv.end());
                return p;
            };
            prompt = pack("context", "pooled");
            if (emb.count("negative_context") && emb.count("negative_pooled"))
                negative = pack("negative_context", "negative_pooled");
            auto s = std::make_unique<mkb::image::Sdxl>(c);
            if (random) {
                s->init_random(o.weights_seed);
            } else {
                const auto files = part_files(pos[0], {"unet"});
                std::vector<const char*> p;
                for (const auto& f : files)
                    p.push_back(f.c_str());
                check(mkb_unet_load_safetensors(s->handle(), p.data(), int(p.size()), 1, nullptr), "unet");
            }
            if (!o.lora.empty())
                check(mkb_unet_load_lora(s->handle(), o.lora.c_str(), o.lora_scale, nullptr), "lora");
            engine = std::move(s);
        }

        for (uint32_t n = 0; n < o.count; ++n) {
            mkb::image::Engine::Request r;
            r.prompt = prompt;
            r.negative = negative;
            r.h = gh;
            r.w = gw;
            r.steps = o.steps;
            r.guidance = o.guidance;
            r.sampler = o.sampler;
            r.seed = o.seed + n;
            const auto t0 = std::chrono::steady_clock::now();
            const std::vector<float> lat = qimg ? qimg->denoise_device(r) : engine->denoise(r);
            const auto img = vae.decode(lat, gh, gw);
            const double ms =
                std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
            std::string path = o.out;
            if (n > 0) {
                const size_t dot = path.rfind('.');
                path = dot == std::string::npos ? path + "-" + std::to_string(n)
                                                : path.substr(0, dot) + "-" + std::to_string(n) + path.substr(dot);
            }
            mkb::image::Provenance prov;
            prov.prompt = pos[1];
            prov.model = random ? "random-" + o.model : fs::path(pos[0]).lexically_normal().filename().string();
            const float g = o.guidance.value_or(engine->default_guidance());
            const bool guided = !negative.empty() && g != 1.0f;
            if (guided)
                prov.negative = std::string("(embeddings)");
            prov.guidance = guided ? g : 1.0f;
            prov.sampler = mkb::image::sampler_name(o.sampler.value_or(engine->default_sampler()));
            prov.steps = o.steps ? o.steps : engine->default_steps();
            prov.width = o.width;
            prov.height = o.height;
            prov.seed = r.seed;
            if (!o.lora.empty())
                prov.loras.push_back({fs::path(o.lora).stem().string(), o.lora_scale});
            mkb::image::write_file(
                path, mkb::image::with_provenance(
                          mkb::image::encode_png(mkb::image::to_rgba8(img), o.width, o.height, o.rgb), prov));
            if (!o.latents_out.empty() && n == 0)
                mkb::image::write_file(o.latents_out,
                                       std::span<const uint8_t>(reinterpret_cast<const uint8_t*>(lat.data()),
                                                                lat.size() * 4));
            std::printf("%ux%u, %u steps in %.1f ms: %s\n", o.width, o.height, prov.steps, ms, path.c_str());
        }
    } catch (const std::exception& e) {
        std::fprintf(stderr, "mako_image: %s\n%s", e.what(), pos.size() == 2 ? "" : kUsage);
        return 1;
    }
    return 0;
}
