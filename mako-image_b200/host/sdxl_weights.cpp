// SDXL UNet and VAE decoder weights from safetensors checkpoints (include/mkb_image.h, "Weights from files").
//
// The reference loads the UNet under the original (SGM) checkpoint names, "model.diffusion_model.input_blocks.4.1.
// transformer_blocks.0.attn1.to_q.weight" and so on (Sdxl::load_unet / load_res / load_trans,
// src/image/sdxl.cpp:238-362: q/k/v and cross k/v row-stacked), and the VAE decoder under the Diffusers names with the
// original AutoencoderKL names as the alternative (Engine::load_vae_kl and ldm_name, src/image/engine.cpp:92-118,
// 590-640). Each of the handle's weights (named by block position, "in4.attn.b0.qkv.w", "up1.res2.conv1.w") is pulled
// from its source tensors: convolutions go from the checkpoint's [out][in][ky][kx] to the table's [out][ky][kx][in],
// 1x1 convolutions used as matrices are squeezed, stacked rows are concatenated. Tensors the model does not use (a
// single-file checkpoint also holds the text encoders) are ignored.
#include "mkb_image.h"
#include "lora_file.hpp"
#include "safetensors.hpp"

#include <cstdio>
#include <cstring>
#include <functional>
#include <map>
#include <string>
#include <vector>

namespace mkb {
mkb_status fail(mkb_status code, const std::string& msg);  // the library's error reporter (api_ops.cu)
}

namespace {

using mkb::fail;

// Candidate sources of one weight: alternatives in order, each a list of tensors stacked by rows.
using Alts = std::vector<std::vector<std::string>>;

bool take_prefix(const std::string& s, const std::string& pre, std::string* rest)
{
    if (s.rfind(pre, 0) != 0)
        return false;
    *rest = s.substr(pre.size());
    return true;
}

// "x.w" / "x.b" -> ("x", ".weight" / ".bias").
bool split_wb(const std::string& s, std::string* stem, std::string* suf)
{
    if (s.size() > 2 && s.compare(s.size() - 2, 2, ".w") == 0)
        *suf = ".weight";
    else if (s.size() > 2 && s.compare(s.size() - 2, 2, ".b") == 0)
        *suf = ".bias";
    else
        return false;
    *stem = s.substr(0, s.size() - 2);
    return true;
}

// Residual-block parameter of the UNet (sdxl.cpp:238-262).
bool unet_res(const std::string& x, std::string* out)
{
    std::string stem, suf;
    if (!split_wb(x, &stem, &suf))
        return false;
    const std::pair<const char*, const char*> m[] = {{"gn1", "in_layers.0"},  {"conv1", "in_layers.2"},
                                                     {"gn2", "out_layers.0"}, {"conv2", "out_layers.3"},
                                                     {"skip", "skip_connection"}, {"emb", "emb_layers.1"}};
    for (auto& [ours, theirs] : m)
        if (stem == ours) {
            *out = std::string(theirs) + suf;
            return true;
        }
    return false;
}

// Transformer parameter of the UNet (sdxl.cpp:264-310), relative to the transformer's prefix.
bool unet_attn(const std::string& x, Alts* alts)
{
    std::string stem, suf;
    if (!split_wb(x, &stem, &suf))
        return false;
    for (auto [ours, theirs] : {std::pair<const char*, const char*>{"gn", "norm"}, {"proj_in", "proj_in"},
                                {"proj_out", "proj_out"}})
        if (stem == ours) {
            *alts = {{std::string(theirs) + suf}};
            return true;
        }
    unsigned j = 0;
    int used = 0;
    if (std::sscanf(stem.c_str(), "b%u.%n", &j, &used) != 1 || used <= 0)
        return false;
    const std::string tb = "transformer_blocks." + std::to_string(j) + ".", rest = stem.substr(size_t(used));
    if (rest == "qkv") {
        *alts = {{tb + "attn1.to_q" + suf, tb + "attn1.to_k" + suf, tb + "attn1.to_v" + suf}};
        return true;
    }
    if (rest == "kv2") {
        *alts = {{tb + "attn2.to_k" + suf, tb + "attn2.to_v" + suf}};
        return true;
    }
    const std::pair<const char*, const char*> m[] = {{"ln1", "norm1"},         {"ln2", "norm2"},
                                                     {"ln3", "norm3"},         {"o1", "attn1.to_out.0"},
                                                     {"q2", "attn2.to_q"},     {"o2", "attn2.to_out.0"},
                                                     {"ff1", "ff.net.0.proj"}, {"ff2", "ff.net.2"}};
    for (auto& [ours, theirs] : m)
        if (rest == ours) {
            *alts = {{tb + theirs + suf}};
            return true;
        }
    return false;
}

// The UNet weight `w` -> its source tensors, without the "model.diffusion_model." prefix.
bool unet_sources(const std::string& w, Alts* alts)
{
    std::string rest, stem, suf;
    const std::pair<const char*, const char*> top[] = {{"conv_in", "input_blocks.0.0"}, {"time.lin1", "time_embed.0"},
                                                       {"time.lin2", "time_embed.2"},   {"label.lin1", "label_emb.0.0"},
                                                       {"label.lin2", "label_emb.0.2"}, {"out.gn", "out.0"},
                                                       {"out.conv", "out.2"}};
    if (split_wb(w, &stem, &suf))
        for (auto& [ours, theirs] : top)
            if (stem == ours) {
                *alts = {{std::string(theirs) + suf}};
                return true;
            }
    unsigned k = 0;
    int used = 0;
    std::string blk, part;
    if (std::sscanf(w.c_str(), "in%u.%n", &k, &used) == 1 && used > 0) {
        blk = "input_blocks." + std::to_string(k) + ".";
    } else if (used = 0; std::sscanf(w.c_str(), "out%u.%n", &k, &used) == 1 && used > 0) {
        blk = "output_blocks." + std::to_string(k) + ".";
    } else if (take_prefix(w, "mid.res0.", &rest)) {
        std::string r;
        if (!unet_res(rest, &r))
            return false;
        *alts = {{"middle_block.0." + r}};
        return true;
    } else if (take_prefix(w, "mid.res1.", &rest)) {
        std::string r;
        if (!unet_res(rest, &r))
            return false;
        *alts = {{"middle_block.2." + r}};
        return true;
    } else if (take_prefix(w, "mid.attn.", &rest)) {
        Alts a;
        if (!unet_attn(rest, &a))
            return false;
        for (auto& set : a)
            for (auto& n : set)
                n = "middle_block.1." + n;
        *alts = a;
        return true;
    } else {
        return false;
    }
    rest = w.substr(size_t(used));
    std::string r;
    if (take_prefix(rest, "res.", &part) && unet_res(part, &r)) {
        *alts = {{blk + "0." + r}};
        return true;
    }
    if (split_wb(rest, &stem, &suf) && stem == "down") {
        *alts = {{blk + "0.op" + suf}};
        return true;
    }
    if (split_wb(rest, &stem, &suf) && stem == "up") {  // after the block's transformer, or its residual block
        *alts = {{blk + "2.conv" + suf}, {blk + "1.conv" + suf}};
        return true;
    }
    if (take_prefix(rest, "attn.", &part)) {
        Alts a;
        if (!unet_attn(part, &a))
            return false;
        for (auto& set : a)
            for (auto& n : set)
                n = blk + "1." + n;
        *alts = a;
        return true;
    }
    return false;
}

// The VAE decoder weight `w` -> Diffusers names, then the original AutoencoderKL names (engine.cpp:92-118).
bool vae_sources(const std::string& w, Alts* alts)
{
    std::string stem, suf, rest;
    if (!split_wb(w, &stem, &suf))
        return false;
    auto res = [&](const std::string& r, std::string* d, std::string* o) {
        const std::pair<const char*, const char*> m[] = {{"gn1", "norm1"}, {"conv1", "conv1"}, {"gn2", "norm2"},
                                                         {"conv2", "conv2"}};
        for (auto& [ours, theirs] : m)
            if (r == ours) {
                *d = *o = theirs;
                return true;
            }
        if (r == "skip") {
            *d = "conv_shortcut";
            *o = "nin_shortcut";
            return true;
        }
        return false;
    };
    const std::pair<const char*, const char*> top[][3] = {
        {{"post_quant", ""}, {"post_quant_conv", ""}, {"post_quant_conv", ""}},
        {{"conv_in", ""}, {"decoder.conv_in", ""}, {"decoder.conv_in", ""}},
        {{"out.gn", ""}, {"decoder.conv_norm_out", ""}, {"decoder.norm_out", ""}},
        {{"out.conv", ""}, {"decoder.conv_out", ""}, {"decoder.conv_out", ""}},
        {{"mid.attn.gn", ""}, {"decoder.mid_block.attentions.0.group_norm", ""}, {"decoder.mid.attn_1.norm", ""}},
        {{"mid.attn.proj", ""}, {"decoder.mid_block.attentions.0.to_out.0", ""}, {"decoder.mid.attn_1.proj_out", ""}}};
    for (const auto& t : top)
        if (stem == t[0].first) {
            *alts = {{std::string(t[1].first) + suf}, {std::string(t[2].first) + suf}};
            return true;
        }
    if (stem == "mid.attn.qkv") {
        const std::string d = "decoder.mid_block.attentions.0.", o = "decoder.mid.attn_1.";
        *alts = {{d + "to_q" + suf, d + "to_k" + suf, d + "to_v" + suf}, {o + "q" + suf, o + "k" + suf, o + "v" + suf}};
        return true;
    }
    std::string d, o;
    for (int m = 0; m < 2; ++m)
        if (take_prefix(stem, m ? "mid.res1." : "mid.res0.", &rest) && res(rest, &d, &o)) {
            *alts = {{"decoder.mid_block.resnets." + std::to_string(m) + "." + d + suf},
                     {"decoder.mid.block_" + std::to_string(m + 1) + "." + o + suf}};
            return true;
        }
    unsigned i = 0, k = 0;
    int used = 0;
    constexpr unsigned kLevels = 4;
    if (std::sscanf(stem.c_str(), "up%u.res%u.%n", &i, &k, &used) == 2 && used > 0 && i < kLevels &&
        res(stem.substr(size_t(used)), &d, &o)) {
        *alts = {{"decoder.up_blocks." + std::to_string(i) + ".resnets." + std::to_string(k) + "." + d + suf},
                 {"decoder.up." + std::to_string(kLevels - 1 - i) + ".block." + std::to_string(k) + "." + o + suf}};
        return true;
    }
    if (used = 0; std::sscanf(stem.c_str(), "up%u.up%n", &i, &used) == 1 && used == int(stem.size()) && i < kLevels) {
        *alts = {{"decoder.up_blocks." + std::to_string(i) + ".upsamplers.0.conv" + suf},
                 {"decoder.up." + std::to_string(kLevels - 1 - i) + ".upsample.conv" + suf}};
        return true;
    }
    return false;
}

// The text encoders' weights (Sdxl::load_clip, src/image/sdxl.cpp:154-237): ViT-L in the HF CLIPTextModel names
// (q, k, v projections stacked into qkv), bigG in the OpenCLIP names (in_proj already stacked).
bool clip_sources(int which, const std::string& w, Alts* alts)
{
    if (w == "tok" || w == "pos") {
        const bool t = w == "tok";
        *alts = {{which == 0 ? (t ? "embeddings.token_embedding.weight" : "embeddings.position_embedding.weight")
                             : (t ? "token_embedding.weight" : "positional_embedding")}};
        return true;
    }
    if (which == 1 && (w == "lnf.w" || w == "lnf.b" || w == "proj")) {
        *alts = {{w == "proj" ? "text_projection" : w == "lnf.w" ? "ln_final.weight" : "ln_final.bias"}};
        return true;
    }
    unsigned i = 0;
    int used = 0;
    if (std::sscanf(w.c_str(), "l%u.%n", &i, &used) != 1 || used <= 0)
        return false;
    std::string stem, suf;
    if (!split_wb(w.substr(size_t(used)), &stem, &suf))
        return false;
    const std::string n = std::to_string(i);
    if (which == 0) {
        const std::string l = "encoder.layers." + n + ".";
        if (stem == "qkv") {
            *alts = {{l + "self_attn.q_proj" + suf, l + "self_attn.k_proj" + suf, l + "self_attn.v_proj" + suf}};
            return true;
        }
        const std::pair<const char*, const char*> m[] = {{"ln1", "layer_norm1"}, {"o", "self_attn.out_proj"},
                                                         {"ln2", "layer_norm2"}, {"fc1", "mlp.fc1"},
                                                         {"fc2", "mlp.fc2"}};
        for (auto& [ours, theirs] : m)
            if (stem == ours) {
                *alts = {{l + theirs + suf}};
                return true;
            }
        return false;
    }
    const std::string l = "transformer.resblocks." + n + ".";
    if (stem == "qkv") {
        *alts = {{l + (suf == ".weight" ? "attn.in_proj_weight" : "attn.in_proj_bias")}};
        return true;
    }
    const std::pair<const char*, const char*> m[] = {{"ln1", "ln_1"}, {"o", "attn.out_proj"}, {"ln2", "ln_2"},
                                                     {"fc1", "mlp.c_fc"}, {"fc2", "mlp.c_proj"}};
    for (auto& [ours, theirs] : m)
        if (stem == ours) {
            *alts = {{l + theirs + suf}};
            return true;
        }
    return false;
}

}  // namespace

namespace {

struct Model {
    std::function<int()> count;
    std::function<mkb_status(int, const char**, long*, int*)> info;
    std::function<mkb_status(const char*, const float*)> write;
    std::function<bool(const std::string&, Alts*)> sources;
    std::vector<std::string> prefixes;  // tried in order in front of every source name
    const char* what;
};

struct Found {
    const mkb::st::File* f;
    const mkb::st::Tensor* t;
};

mkb_status load(const Model& m, const char* const* paths, int n_paths, int strict, int* loaded)
{
    if (!paths || n_paths < 1)
        return fail(MKB_ERR_INVALID, std::string(m.what) + ": no files");
    std::vector<std::unique_ptr<mkb::st::File>> files;
    std::map<std::string, Found> index;
    for (int i = 0; i < n_paths; ++i) {
        std::string err;
        auto f = mkb::st::File::open(paths[i] ? paths[i] : "", &err);
        if (!f)
            return fail(MKB_ERR_INVALID, err);
        for (const auto& t : f->tensors())
            index.emplace(t.name, Found{f.get(), &t});
        files.push_back(std::move(f));
    }
    auto lookup = [&](const std::string& n) -> const Found* {
        for (const auto& pre : m.prefixes) {
            auto it = index.find(pre + n);
            if (it != index.end())
                return &it->second;
        }
        return nullptr;
    };
    int count = 0;
    std::vector<float> buf, tmp;
    for (int wi = 0; wi < m.count(); ++wi) {
        const char* name = nullptr;
        long dims[4] = {0, 0, 0, 0};
        int nd = 0;
        if (mkb_status s = m.info(wi, &name, dims, &nd); s != MKB_OK)
            return s;
        Alts alts;
        if (!m.sources(name, &alts))
            return fail(MKB_ERR_INVALID, std::string(m.what) + ": no checkpoint name for " + name);
        std::vector<const Found*> src;
        for (const auto& set : alts) {
            src.clear();
            for (const auto& n : set)
                if (const Found* f = lookup(n))
                    src.push_back(f);
            if (src.size() == set.size())
                break;
            src.clear();
        }
        if (src.empty()) {
            if (strict)
                return fail(MKB_ERR_INVALID, std::string(m.what) + ": the files lack " + name + " (" +
                                                 alts.front().front() + ")");
            continue;
        }
        // The table's logical layout: [r], [r][c] or a 3x3 convolution [r][3][3][c].
        const long rows = dims[0], cols = nd == 1 ? 1 : nd == 4 ? dims[3] : dims[1];
        const long per_row = nd == 4 ? 9 * cols : cols;
        buf.assign(size_t(rows) * per_row, 0.f);
        long r0 = 0;
        for (const Found* fd : src) {
            const auto& sh = fd->t->shape;
            const bool conv3 = nd == 4 && sh.size() == 4 && sh[1] == cols && sh[2] == 3 && sh[3] == 3;
            const bool mat = nd == 2 && ((sh.size() == 2 && sh[1] == cols) ||
                                         (sh.size() == 4 && sh[1] == cols && sh[2] == 1 && sh[3] == 1));
            const bool vec = nd == 1 && sh.size() == 1;
            if (!(conv3 || mat || vec) || sh.empty() || r0 + sh[0] > rows)
                return fail(MKB_ERR_INVALID, std::string(m.what) + ": " + fd->t->name + " does not fit " + name);
            std::string err;
            tmp.resize(size_t(fd->t->count()));
            if (!fd->f->read_f32(*fd->t, tmp.data(), &err))
                return fail(MKB_ERR_INVALID, err);
            if (conv3) {  // [out][in][ky][kx] -> [out][ky][kx][in]
                for (long o = 0; o < sh[0]; ++o)
                    for (long c = 0; c < cols; ++c)
                        for (int k = 0; k < 9; ++k)
                            buf[size_t(r0 + o) * per_row + size_t(k) * cols + c] = tmp[(size_t(o) * cols + c) * 9 + k];
            } else {
                std::memcpy(buf.data() + size_t(r0) * per_row, tmp.data(), tmp.size() * 4);
            }
            r0 += sh[0];
        }
        if (r0 != rows)
            return fail(MKB_ERR_INVALID, std::string(m.what) + ": the sources of " + name + " have " +
                                             std::to_string(r0) + " rows, it needs " + std::to_string(rows));
        if (mkb_status s = m.write(name, buf.data()); s != MKB_OK)
            return s;
        ++count;
    }
    if (loaded)
        *loaded = count;
    return MKB_OK;
}

}  // namespace

extern "C" {

mkb_status mkb_unet_load_safetensors(mkb_unet* u, const char* const* paths, int n_paths, int strict, int* loaded)
{
    if (!u)
        return fail(MKB_ERR_INVALID, "unet: null handle");
    Model m{[u] { return mkb_unet_weight_count(u); },
            [u](int i, const char** n, long* d, int* nd) { return mkb_unet_weight_info(u, i, n, d, nd); },
            [u](const char* n, const float* h) { return mkb_unet_weight_write(u, n, h); },
            unet_sources,
            {"model.diffusion_model.", ""},
            "unet"};
    return load(m, paths, n_paths, strict, loaded);
}

mkb_status mkb_clip_load_safetensors(mkb_clip* c, const char* const* paths, int n_paths, int strict, int* loaded)
{
    if (!c)
        return fail(MKB_ERR_INVALID, "clip: null handle");
    int which = 0;
    for (int i = 0; i < mkb_clip_weight_count(c); ++i) {  // bigG's table alone has the text projection
        const char* n = nullptr;
        if (mkb_clip_weight_info(c, i, &n, nullptr, nullptr) == MKB_OK && std::strcmp(n, "proj") == 0)
            which = 1;
    }
    Model m{[c] { return mkb_clip_weight_count(c); },
            [c](int i, const char** n, long* d, int* nd) { return mkb_clip_weight_info(c, i, n, d, nd); },
            [c](const char* n, const float* h) { return mkb_clip_weight_write(c, n, h); },
            [which](const std::string& w, Alts* a) { return clip_sources(which, w, a); },
            which == 0 ? std::vector<std::string>{"conditioner.embedders.0.transformer.text_model.", "text_model.", ""}
                       : std::vector<std::string>{"conditioner.embedders.1.model.", ""},
            "clip"};
    return load(m, paths, n_paths, strict, loaded);
}

mkb_status mkb_vae_load_safetensors(mkb_vae* v, const char* const* paths, int n_paths, int strict, int* loaded)
{
    if (!v)
        return fail(MKB_ERR_INVALID, "vae: null handle");
    Model m{[v] { return mkb_vae_weight_count(v); },
            [v](int i, const char** n, long* d, int* nd) { return mkb_vae_weight_info(v, i, n, d, nd); },
            [v](const char* n, const float* h) { return mkb_vae_weight_write(v, n, h); },
            vae_sources,
            {"", "first_stage_model.", "vae."},
            "vae"};
    return load(m, paths, n_paths, strict, loaded);
}

}  // extern "C"

namespace {

// A UNet LoRA module -> (weight, first row, rows): the transformers' projections, as Sdxl::load_unet registers them
// (sdxl.cpp:385-410). Names compare with '_' read as '.' (the reference's lora_key, sdxl.cpp:54-58), so the
// checkpoint spelling ("input_blocks.4.1.transformer_blocks.0.attn1.to_q") and the flattened one of many adapter
// files ("input_blocks_4_1_transformer_blocks_0_attn1_to_q") both resolve.
bool unet_lora_target(const std::string& module, const std::map<std::string, std::vector<long>>& dims,
                      std::string* weight, long* row0, long* rows)
{
    std::string m = module;
    for (char& ch : m)
        if (ch == '_')
            ch = '.';
    unsigned k = 0, j = 0;
    int used = 0;
    std::string base, rest;
    if (std::sscanf(m.c_str(), "input.blocks.%u.1.%n", &k, &used) == 1 && used > 0)
        base = "in" + std::to_string(k) + ".attn.";
    else if (used = 0; std::sscanf(m.c_str(), "output.blocks.%u.1.%n", &k, &used) == 1 && used > 0)
        base = "out" + std::to_string(k) + ".attn.";
    else if (used = 0; m.rfind("middle.block.1.", 0) == 0)
        base = "mid.attn.", used = int(std::strlen("middle.block.1."));
    else
        return false;
    rest = m.substr(size_t(used));
    auto whole = [&](const std::string& w) {
        const auto it = dims.find(w);
        if (it == dims.end())
            return false;
        *weight = w;
        *row0 = 0;
        *rows = it->second[0];
        return true;
    };
    if (rest == "proj.in")
        return whole(base + "proj_in.w");
    if (rest == "proj.out")
        return whole(base + "proj_out.w");
    used = 0;
    if (std::sscanf(rest.c_str(), "transformer.blocks.%u.%n", &j, &used) != 1 || used <= 0)
        return false;
    const std::string b = base + "b" + std::to_string(j) + ".", what = rest.substr(size_t(used));
    const auto o1 = dims.find(b + "o1.w");
    if (o1 == dims.end())
        return false;
    const long c = o1->second[0];
    struct Part {
        const char* name;
        const char* weight;
        long row0, rows;  // in units of c; rows 0: the whole matrix
    };
    const Part parts[] = {{"attn1.to.q", "qkv.w", 0, 1},    {"attn1.to.k", "qkv.w", 1, 1},
                          {"attn1.to.v", "qkv.w", 2, 1},    {"attn1.to.out.0", "o1.w", 0, 0},
                          {"attn2.to.q", "q2.w", 0, 0},     {"attn2.to.k", "kv2.w", 0, 1},
                          {"attn2.to.v", "kv2.w", 1, 1},    {"attn2.to.out.0", "o2.w", 0, 0},
                          {"ff.net.0.proj", "ff1.w", 0, 0}, {"ff.net.2", "ff2.w", 0, 0}};
    for (const Part& p : parts)
        if (what == p.name) {
            if (!whole(b + p.weight))
                return false;
            if (p.rows) {
                *row0 = p.row0 * c;
                *rows = p.rows * c;
            }
            return true;
        }
    return false;
}

std::map<std::string, std::vector<long>> unet_dims(const mkb_unet* u)
{
    std::map<std::string, std::vector<long>> out;
    for (int i = 0; i < mkb_unet_weight_count(u); ++i) {
        const char* name = nullptr;
        long d[4] = {0, 0, 0, 0};
        int nd = 0;
        if (mkb_unet_weight_info(u, i, &name, d, &nd) == MKB_OK)
            out[name] = std::vector<long>(d, d + nd);
    }
    return out;
}

mkb_status unet_merge(mkb_unet* u, const std::map<std::string, std::vector<long>>& dims, const std::string& module,
                      const float* A, const float* B, int rank, int in, int out, float scale)
{
    std::string w;
    long row0 = 0, rows = 0;
    if (!unet_lora_target(module, dims, &w, &row0, &rows))
        return fail(MKB_ERR_INVALID, "unet lora: " + module + " is not a projection of this UNet");
    const auto& d = dims.at(w);
    if (d.size() != 2 || in != d[1] || out != rows)
        return fail(MKB_ERR_INVALID, "unet lora: " + module + " is " + std::to_string(rows) + " x " +
                                         std::to_string(d.size() == 2 ? d[1] : 0) + ", the adapter " +
                                         std::to_string(out) + " x " + std::to_string(in));
    return mkb_unet_weight_lora_rows(u, w.c_str(), row0, rows, A, B, rank, scale);
}

}  // namespace

extern "C" {

mkb_status mkb_unet_lora_merge(mkb_unet* u, const char* module, const float* A, const float* B, int rank,
                               int in_features, int out_features, float scale)
{
    if (!u || !module || !A || !B)
        return fail(MKB_ERR_INVALID, "unet lora: null argument");
    return unet_merge(u, unet_dims(u), module, A, B, rank, in_features, out_features, scale);
}

mkb_status mkb_unet_load_lora(mkb_unet* u, const char* path, float scale, int* merged)
{
    if (!u)
        return fail(MKB_ERR_INVALID, "unet lora: null handle");
    const auto dims = unet_dims(u);
    return mkb::load_lora_file(
        path, scale,
        [u, &dims](const std::string& m, const float* A, const float* B, int r, int in, int out, float s) {
            return unet_merge(u, dims, m, A, B, r, in, out, s);
        },
        merged);
}

}  // extern "C"
