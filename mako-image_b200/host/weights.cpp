// Checkpoints and LoRA adapters into the denoiser handle (include/mkb_image.h, "Weights from files").
//
// The reference loads its transformer from safetensors files and stacks q/k/v and gate/up rows into single matrices
// (QwenImage::load_transformer, src/image/qwen_image.cpp:79-111); LoRA adapters are added by module name, each module
// resolving to a row range of one of those matrices (QwenImage::lora_target, qwen_image.cpp:295-331). This file
// maps checkpoint tensor names onto the handle's weight table the same way, for both block variants: MKB_VARIANT_REF21
// uses the reference's names, MKB_VARIANT_QWEN1 the published Qwen-Image transformer's (separate image / text stream
// weights, biases, per-block modulation).
#include "mkb_image.h"
#include "lora_file.hpp"
#include "safetensors.hpp"

#include <cstdio>
#include <cstring>
#include <map>
#include <set>
#include <string>
#include <vector>

namespace mkb {
mkb_status fail(mkb_status code, const std::string& msg);  // the library's error reporter (api_ops.cu)
}

namespace {

using mkb::fail;

// Where a checkpoint tensor goes: rows [row0, row0 + rows) of the handle's weight `weight` (rows 0: all of them).
struct Target {
    std::string weight;
    long row0 = 0, rows = 0;
    bool plus_one = false;  // stored zero-centred: the scale is the stored value + 1
};

struct Shape {
    int variant = -1;
    long D = 0, F = 0;
    int blocks = 0;
};

bool ends_with(const std::string& s, const char* suf, std::string* stem)
{
    const size_t n = std::strlen(suf);
    if (s.size() < n || s.compare(s.size() - n, n, suf) != 0)
        return false;
    *stem = s.substr(0, s.size() - n);
    return true;
}

// Module (a tensor name without ".weight" / ".bias") of the reference's variant -> target. Row ranges follow
// qwen_image.cpp:295-331.
bool ref21_module(const Shape& sh, const std::string& m, bool bias, Target* t)
{
    if (bias)
        return false;  // the reference's transformer has no biases
    unsigned b = 0;
    int used = 0;
    if (std::sscanf(m.c_str(), "transformer_blocks.%u.%n", &b, &used) == 1 && used > 0) {
        if (int(b) >= sh.blocks)
            return false;
        const std::string p = "blk" + std::to_string(b) + ".", rest = m.substr(size_t(used));
        const long D = sh.D, F = sh.F;
        struct Row {
            const char* name;
            const char* weight;
            long row0, rows;
        };
        const Row rows[] = {{"attn.to_q", "qkv.w", 0, D},          {"attn.to_k", "qkv.w", D, D},
                            {"attn.to_v", "qkv.w", 2 * D, D},      {"attn.to_out.0", "o.w", 0, D},
                            {"attn.norm_q", "norm_q", 0, 0},       {"attn.norm_k", "norm_k", 0, 0},
                            {"img_mlp.gate_layer", "gate_up.w", 0, F}, {"img_mlp.proj", "gate_up.w", F, F},
                            {"img_mlp.gate_up", "gate_up.w", 0, 2 * F}, {"img_mlp.out", "down.w", 0, D}};
        for (const Row& r : rows)
            if (rest == r.name) {
                *t = Target{p + r.weight, r.row0, r.rows, false};
                return true;
            }
        return false;
    }
    const std::pair<const char*, const char*> top[] = {
        {"img_in", "img_in.w"},
        {"txt_in.in_layer", "txt_in1.w"},
        {"txt_in.out_layer", "txt_in2.w"},
        {"time_text_embed.timestep_embedder.linear_1", "time.lin1.w"},
        {"time_text_embed.timestep_embedder.linear_2", "time.lin2.w"},
        {"modulation.1", "mod.w"},
        {"norm_out.linear", "norm_out.w"},
        {"proj_out", "proj_out.w"}};
    for (auto& [ck, w] : top)
        if (m == ck) {
            *t = Target{w, 0, 0, false};
            return true;
        }
    if (m == "txt_in.text_norm") {  // stored zero-centred (qwen_image.cpp:83-87)
        *t = Target{"txt_norm.w", 0, 0, true};
        return true;
    }
    return false;
}

// Module of the Qwen-Image variant (image and text streams, biases) -> target.
bool qwen1_module(const Shape& sh, const std::string& m, bool bias, Target* t)
{
    const char* wb = bias ? "b" : "w";
    unsigned b = 0;
    int used = 0;
    if (std::sscanf(m.c_str(), "transformer_blocks.%u.%n", &b, &used) == 1 && used > 0) {
        if (int(b) >= sh.blocks)
            return false;
        const std::string p = "blk" + std::to_string(b) + ".", rest = m.substr(size_t(used));
        const long D = sh.D;
        struct Row {
            const char* name;
            const char* stream;
            const char* weight;  // without the .w / .b suffix
            long row0, rows;
            bool has_bias;
        };
        const Row rows[] = {{"img_mod.1", "img", "mod", 0, 0, true},
                            {"txt_mod.1", "txt", "mod", 0, 0, true},
                            {"attn.to_q", "img", "qkv", 0, D, true},
                            {"attn.to_k", "img", "qkv", D, D, true},
                            {"attn.to_v", "img", "qkv", 2 * D, D, true},
                            {"attn.add_q_proj", "txt", "qkv", 0, D, true},
                            {"attn.add_k_proj", "txt", "qkv", D, D, true},
                            {"attn.add_v_proj", "txt", "qkv", 2 * D, D, true},
                            {"attn.to_out.0", "img", "o", 0, 0, true},
                            {"attn.to_add_out", "txt", "o", 0, 0, true},
                            {"img_mlp.net.0.proj", "img", "ff1", 0, 0, true},
                            {"img_mlp.net.2", "img", "ff2", 0, 0, true},
                            {"txt_mlp.net.0.proj", "txt", "ff1", 0, 0, true},
                            {"txt_mlp.net.2", "txt", "ff2", 0, 0, true}};
        for (const Row& r : rows)
            if (rest == r.name) {
                if (bias && !r.has_bias)
                    return false;
                *t = Target{p + r.stream + "." + r.weight + "." + wb, r.row0, r.rows, false};
                return true;
            }
        const std::pair<const char*, const char*> norms[] = {{"attn.norm_q", "img.norm_q"},
                                                             {"attn.norm_k", "img.norm_k"},
                                                             {"attn.norm_added_q", "txt.norm_q"},
                                                             {"attn.norm_added_k", "txt.norm_k"}};
        for (auto& [ck, w] : norms)
            if (rest == ck && !bias) {
                *t = Target{p + w, 0, 0, false};
                return true;
            }
        return false;
    }
    const std::pair<const char*, const char*> top[] = {{"img_in", "img_in"},
                                                       {"txt_in", "txt_in"},
                                                       {"time_text_embed.timestep_embedder.linear_1", "time.lin1"},
                                                       {"time_text_embed.timestep_embedder.linear_2", "time.lin2"},
                                                       {"norm_out.linear", "norm_out"},
                                                       {"proj_out", "proj_out"}};
    for (auto& [ck, w] : top)
        if (m == ck) {
            *t = Target{std::string(w) + "." + wb, 0, 0, false};
            return true;
        }
    if (m == "txt_norm" && !bias) {
        *t = Target{"txt_norm.w", 0, 0, false};
        return true;
    }
    return false;
}

// A checkpoint tensor name ("<module>.weight" / "<module>.bias") -> target.
bool tensor_target(const Shape& sh, const std::string& name, Target* t)
{
    std::string stem;
    bool bias = false;
    if (ends_with(name, ".weight", &stem))
        bias = false;
    else if (ends_with(name, ".bias", &stem))
        bias = true;
    else
        return false;
    return sh.variant == MKB_VARIANT_REF21 ? ref21_module(sh, stem, bias, t) : qwen1_module(sh, stem, bias, t);
}

}  // namespace

namespace {

struct Table {
    Shape shape;
    std::map<std::string, std::pair<long, long>> dims;  // weight -> (rows, cols); cols 0 for vectors
};

mkb_status read_table(const mkb_dit* d, Table* tb)
{
    tb->shape.variant = mkb_dit_variant(d);
    if (tb->shape.variant < 0)
        return fail(MKB_ERR_INVALID, "weights: null handle");
    const int n = mkb_dit_weight_count(d);
    for (int i = 0; i < n; ++i) {
        const char* name = nullptr;
        long r = 0, c = 0;
        if (mkb_dit_weight_info(d, i, &name, &r, &c) != MKB_OK)
            return MKB_ERR_INVALID;
        tb->dims[name] = {r, c};
    }
    const auto img_in = tb->dims.find("img_in.w");
    if (img_in == tb->dims.end())
        return fail(MKB_ERR_INVALID, "weights: handle without img_in.w");
    tb->shape.D = img_in->second.first;
    const bool q1 = tb->shape.variant == MKB_VARIANT_QWEN1;
    const auto ff = tb->dims.find(q1 ? "blk0.img.ff1.w" : "blk0.down.w");
    if (ff == tb->dims.end())
        return fail(MKB_ERR_INVALID, "weights: handle without blocks");
    tb->shape.F = q1 ? ff->second.first : ff->second.second;
    while (tb->dims.count("blk" + std::to_string(tb->shape.blocks) + (q1 ? ".img.o.w" : ".o.w")))
        ++tb->shape.blocks;
    return MKB_OK;
}

std::string shape_str(const std::vector<int64_t>& s)
{
    std::string o = "[";
    for (size_t i = 0; i < s.size(); ++i)
        o += (i ? ", " : "") + std::to_string(s[i]);
    return o + "]";
}

// Rows and columns a tensor must have to fill target t of table tb (cols 0: a vector).
bool target_dims(const Table& tb, const Target& t, long* rows, long* cols)
{
    const auto it = tb.dims.find(t.weight);
    if (it == tb.dims.end())
        return false;
    *rows = t.rows ? t.rows : it->second.first;
    *cols = it->second.second;
    return t.row0 + *rows <= it->second.first;
}

}  // namespace

extern "C" {

mkb_status mkb_dit_load_safetensors(mkb_dit* d, const char* const* paths, int n_paths, int strict, int* loaded)
{
    if (!d || !paths || n_paths < 1)
        return fail(MKB_ERR_INVALID, "load_safetensors: bad arguments");
    Table tb;
    if (mkb_status s = read_table(d, &tb); s != MKB_OK)
        return s;
    std::map<std::string, long> rows_written;
    std::vector<float> buf;
    int count = 0;
    for (int fi = 0; fi < n_paths; ++fi) {
        std::string err;
        auto f = mkb::st::File::open(paths[fi] ? paths[fi] : "", &err);
        if (!f)
            return fail(MKB_ERR_INVALID, err);
        for (const auto& t : f->tensors()) {
            Target tg;
            if (!tensor_target(tb.shape, t.name, &tg)) {
                if (strict)
                    return fail(MKB_ERR_INVALID, "load_safetensors: " + t.name + " (in " + f->path() +
                                                     ") matches no weight of this model");
                continue;
            }
            long rows = 0, cols = 0;
            if (!target_dims(tb, tg, &rows, &cols))
                return fail(MKB_ERR_INVALID, "load_safetensors: " + t.name + " has no place in " + tg.weight);
            const bool shape_ok = cols ? (t.shape.size() == 2 && t.shape[0] == rows && t.shape[1] == cols)
                                       : (t.shape.size() == 1 && t.shape[0] == rows);
            if (!shape_ok)
                return fail(MKB_ERR_INVALID, "load_safetensors: " + t.name + " is " + shape_str(t.shape) + ", " +
                                                 tg.weight + " needs " +
                                                 (cols ? shape_str({rows, cols}) : shape_str({rows})));
            buf.resize(size_t(t.count()));
            if (!f->read_f32(t, buf.data(), &err))
                return fail(MKB_ERR_INVALID, err);
            if (tg.plus_one)
                for (float& v : buf)
                    v += 1.0f;
            if (mkb_status s = mkb_dit_weight_write_rows(d, tg.weight.c_str(), tg.row0, rows, buf.data());
                s != MKB_OK)
                return s;
            rows_written[tg.weight] += rows;
            ++count;
        }
    }
    if (strict)
        for (const auto& [w, rc] : tb.dims)
            if (rows_written[w] != rc.first)
                return fail(MKB_ERR_INVALID, "load_safetensors: the files leave " + w + " (" +
                                                 std::to_string(rc.first - rows_written[w]) + " of " +
                                                 std::to_string(rc.first) + " rows) unwritten");
    if (loaded)
        *loaded = count;
    return MKB_OK;
}

}  // extern "C"

extern "C" {

mkb_status mkb_dit_lora_merge(mkb_dit* d, const char* module, const float* A, const float* B, int rank,
                              int in_features, int out_features, float scale)
{
    if (!d || !module || !A || !B)
        return fail(MKB_ERR_INVALID, "lora_merge: null argument");
    Table tb;
    if (mkb_status s = read_table(d, &tb); s != MKB_OK)
        return s;
    Target tg;
    long rows = 0, cols = 0;
    if (!tensor_target(tb.shape, std::string(module) + ".weight", &tg) || !target_dims(tb, tg, &rows, &cols) || !cols)
        return fail(MKB_ERR_INVALID, std::string("lora_merge: ") + module + " is not a matrix of this model");
    if (in_features != cols || out_features != rows)
        return fail(MKB_ERR_INVALID, std::string("lora_merge: ") + module + " is " + std::to_string(rows) + " x " +
                                         std::to_string(cols) + ", the adapter " + std::to_string(out_features) +
                                         " x " + std::to_string(in_features));
    return mkb_dit_weight_lora_rows(d, tg.weight.c_str(), tg.row0, rows, A, B, rank, scale);
}

mkb_status mkb_dit_load_lora(mkb_dit* d, const char* path, float scale, int* merged)
{
    if (!d)
        return fail(MKB_ERR_INVALID, "load_lora: null handle");
    return mkb::load_lora_file(
        path, scale,
        [d](const std::string& m, const float* A, const float* B, int r, int in, int out, float s) {
            return mkb_dit_lora_merge(d, m.c_str(), A, B, r, in, out, s);
        },
        merged);
}

struct mkb_st_file {
    std::unique_ptr<mkb::st::File> f;
};

mkb_status mkb_st_open(const char* path, mkb_st_file** out)
{
    if (!path || !out)
        return fail(MKB_ERR_INVALID, "st_open: null argument");
    std::string err;
    auto f = mkb::st::File::open(path, &err);
    if (!f)
        return fail(MKB_ERR_INVALID, err);
    *out = new mkb_st_file{std::move(f)};
    return MKB_OK;
}

void mkb_st_close(mkb_st_file* h) { delete h; }

int mkb_st_count(const mkb_st_file* h) { return h ? int(h->f->tensors().size()) : 0; }

mkb_status mkb_st_info(const mkb_st_file* h, int i, const char** name, const char** dtype, int64_t* dims, int* ndim)
{
    if (!h || i < 0 || i >= int(h->f->tensors().size()))
        return fail(MKB_ERR_INVALID, "st_info: index out of range");
    const auto& t = h->f->tensors()[size_t(i)];
    if (t.shape.size() > 8)
        return fail(MKB_ERR_INVALID, "st_info: more than 8 dimensions");
    if (name)
        *name = t.name.c_str();
    if (dtype)
        *dtype = t.dtype_name.c_str();
    if (dims)
        for (size_t k = 0; k < t.shape.size(); ++k)
            dims[k] = t.shape[k];
    if (ndim)
        *ndim = int(t.shape.size());
    return MKB_OK;
}

mkb_status mkb_st_read_f32(const mkb_st_file* h, const char* name, float* out, int64_t count)
{
    if (!h || !name || !out)
        return fail(MKB_ERR_INVALID, "st_read: null argument");
    const auto* t = h->f->find(name);
    if (!t)
        return fail(MKB_ERR_INVALID, std::string("st_read: no tensor ") + name);
    if (t->count() != count)
        return fail(MKB_ERR_INVALID, std::string("st_read: ") + name + " has " + std::to_string(t->count()) +
                                         " elements");
    std::string err;
    if (!h->f->read_f32(*t, out, &err))
        return fail(MKB_ERR_INVALID, err);
    return MKB_OK;
}

}  // extern "C"
