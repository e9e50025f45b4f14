#include "lora_file.hpp"
#include "safetensors.hpp"

#include <cstring>
#include <map>
#include <vector>

namespace mkb {

mkb_status fail(mkb_status code, const std::string& msg);  // the library's error reporter (api_ops.cu)

namespace {

bool ends_with(const std::string& s, const char* suf, std::string* stem)
{
    const size_t n = std::strlen(suf);
    if (s.size() < n || s.compare(s.size() - n, n, suf) != 0)
        return false;
    *stem = s.substr(0, s.size() - n);
    return true;
}

}  // namespace

mkb_status load_lora_file(const char* path, float scale, const LoraMerge& merge, int* merged)
{
    if (!path)
        return fail(MKB_ERR_INVALID, "load_lora: null path");
    std::string err;
    auto f = mkb::st::File::open(path, &err);
    if (!f)
        return fail(MKB_ERR_INVALID, err);
    struct Pair {
        const mkb::st::Tensor *a = nullptr, *b = nullptr, *alpha = nullptr;
    };
    std::map<std::string, Pair> mods;
    for (const auto& t : f->tensors()) {
        std::string name = t.name, stem;
        for (const char* pre : {"transformer.", "diffusion_model.", "base_model.model.", "lora_unet_"})
            if (name.rfind(pre, 0) == 0)
                name = name.substr(std::strlen(pre));
        if (ends_with(name, ".lora_A.weight", &stem) || ends_with(name, ".lora_down.weight", &stem))
            mods[stem].a = &t;
        else if (ends_with(name, ".lora_B.weight", &stem) || ends_with(name, ".lora_up.weight", &stem))
            mods[stem].b = &t;
        else if (ends_with(name, ".alpha", &stem))
            mods[stem].alpha = &t;
        else
            return fail(MKB_ERR_INVALID, "load_lora: " + t.name + " is not a LoRA tensor");
    }
    int n = 0;
    std::vector<float> a, b;
    for (const auto& [m, p] : mods) {
        if (!p.a || !p.b || p.a->shape.size() != 2 || p.b->shape.size() != 2 || p.a->shape[0] != p.b->shape[1])
            return fail(MKB_ERR_INVALID, "load_lora: " + m + " lacks a matching A / B pair");
        const int r = int(p.a->shape[0]);
        float s = scale;
        if (p.alpha) {
            if (p.alpha->count() != 1)
                return fail(MKB_ERR_INVALID, "load_lora: " + m + ".alpha is not a scalar");
            float al = 0.f;
            if (!f->read_f32(*p.alpha, &al, &err))
                return fail(MKB_ERR_INVALID, err);
            s *= al / float(r);
        }
        a.resize(size_t(p.a->count()));
        b.resize(size_t(p.b->count()));
        if (!f->read_f32(*p.a, a.data(), &err) || !f->read_f32(*p.b, b.data(), &err))
            return fail(MKB_ERR_INVALID, err);
        if (mkb_status st = merge(m, a.data(), b.data(), r, int(p.a->shape[1]), int(p.b->shape[0]), s); st != MKB_OK)
            return st;
        ++n;
    }
    if (merged)
        *merged = n;
    return MKB_OK;
}

}  // namespace mkb
