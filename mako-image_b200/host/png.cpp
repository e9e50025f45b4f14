// PNG output (see png.hpp): chunk framing, CRC-32 and Adler-32 by the PNG and zlib specifications (RFC 2083,
// RFC 1950), stored deflate blocks (RFC 1951 section 3.2.4), iTXt text chunks; plus its C ABI entry points.
#include "png.hpp"

#include "../../include/mkb_image.h"

#include <algorithm>
#include <array>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <stdexcept>

namespace mkb {
mkb_status fail(mkb_status code, const std::string& msg);  // the library's error reporter (api_ops.cu)
}

namespace mkb::image {

namespace {

// The reflected CRC-32 polynomial 0xEDB88320, one table entry per byte value.
std::array<uint32_t, 256> crc_table()
{
    std::array<uint32_t, 256> t{};
    for (uint32_t n = 0; n < 256; ++n) {
        uint32_t c = n;
        for (int k = 0; k < 8; ++k)
            c = (c & 1) ? 0xEDB88320u ^ (c >> 1) : c >> 1;
        t[n] = c;
    }
    return t;
}

void put32(std::vector<uint8_t>& o, uint32_t v)
{
    o.push_back(uint8_t(v >> 24));
    o.push_back(uint8_t(v >> 16));
    o.push_back(uint8_t(v >> 8));
    o.push_back(uint8_t(v));
}

// length, type, data, CRC of type + data
void chunk(std::vector<uint8_t>& o, const char type[4], std::span<const uint8_t> data)
{
    put32(o, uint32_t(data.size()));
    const size_t at = o.size();
    o.insert(o.end(), type, type + 4);
    o.insert(o.end(), data.begin(), data.end());
    put32(o, crc32(std::span<const uint8_t>(o.data() + at, 4 + data.size())));
}

std::vector<uint8_t> itxt(const std::string& keyword, const std::string& text)
{
    // keyword, 0, compression flag 0, method 0, empty language tag + 0, empty translated keyword + 0, UTF-8 text
    std::vector<uint8_t> d(keyword.begin(), keyword.end());
    d.insert(d.end(), {0, 0, 0, 0, 0});
    d.insert(d.end(), text.begin(), text.end());
    std::vector<uint8_t> o;
    chunk(o, "iTXt", d);
    return o;
}

std::string json_string(const std::string& s)
{
    std::string o = "\"";
    for (unsigned char c : s) {
        if (c == '"' || c == '\\') {
            o += '\\';
            o += char(c);
        } else if (c < 0x20) {
            char b[8];
            std::snprintf(b, sizeof b, "\\u%04x", c);
            o += b;
        } else {
            o += char(c);
        }
    }
    return o + "\"";
}

std::string num_g(float v)
{
    char b[32];
    std::snprintf(b, sizeof b, "%g", double(v));
    return b;
}

}  // namespace

uint32_t crc32(std::span<const uint8_t> data, uint32_t crc)
{
    static const std::array<uint32_t, 256> table = crc_table();
    uint32_t c = crc ^ 0xFFFFFFFFu;
    for (uint8_t b : data)
        c = table[(c ^ b) & 0xFF] ^ (c >> 8);
    return c ^ 0xFFFFFFFFu;
}

uint32_t adler32(std::span<const uint8_t> data, uint32_t adler)
{
    uint32_t a = adler & 0xFFFF, b = adler >> 16;
    size_t i = 0;
    while (i < data.size()) {
        // 5552 bytes keep both sums below 2^32 before the reduction (zlib's NMAX).
        const size_t n = std::min<size_t>(5552, data.size() - i);
        for (size_t k = 0; k < n; ++k) {
            a += data[i + k];
            b += a;
        }
        a %= 65521;
        b %= 65521;
        i += n;
    }
    return (b << 16) | a;
}

std::vector<uint8_t> to_rgba8(std::span<const float> rgba)
{
    std::vector<uint8_t> out(rgba.size());
    for (size_t i = 0; i < rgba.size(); ++i) {
        const float v = std::fmin(std::fmax(rgba[i] * 0.5f + 0.5f, 0.0f), 1.0f);
        out[i] = uint8_t(std::nearbyint(v * 255.0f));
    }
    return out;
}

std::vector<uint8_t> encode_png(std::span<const uint8_t> rgba8, uint32_t width, uint32_t height, bool rgb)
{
    if (!width || !height || rgba8.size() != size_t(width) * height * 4)
        throw std::runtime_error("encode_png: not width x height RGBA");
    const size_t ch = rgb ? 3 : 4, row = 1 + size_t(width) * ch;
    // The filtered scanlines: filter type 0 (None), then the row's samples.
    std::vector<uint8_t> raw(row * height);
    for (uint32_t y = 0; y < height; ++y) {
        uint8_t* d = raw.data() + y * row;
        d[0] = 0;
        const uint8_t* s = rgba8.data() + size_t(y) * width * 4;
        if (!rgb) {
            std::memcpy(d + 1, s, size_t(width) * 4);
        } else {
            for (uint32_t x = 0; x < width; ++x)
                std::memcpy(d + 1 + x * 3, s + x * 4, 3);
        }
    }
    // zlib: CMF 0x78 (deflate, 32 KB window), FLG 0x01 (check bits: 0x7801 is a multiple of 31), stored blocks of
    // at most 65535 bytes (BFINAL on the last, BTYPE 00, LEN, NLEN), Adler-32 of the raw data.
    std::vector<uint8_t> z = {0x78, 0x01};
    size_t at = 0;
    do {
        const size_t n = std::min<size_t>(65535, raw.size() - at);
        const bool last = at + n == raw.size();
        z.push_back(last ? 1 : 0);
        z.push_back(uint8_t(n & 0xFF));
        z.push_back(uint8_t(n >> 8));
        z.push_back(uint8_t(~n & 0xFF));
        z.push_back(uint8_t((~n >> 8) & 0xFF));
        z.insert(z.end(), raw.begin() + long(at), raw.begin() + long(at + n));
        at += n;
    } while (at < raw.size());
    put32(z, adler32(raw));

    std::vector<uint8_t> png = {0x89, 'P', 'N', 'G', '\r', '\n', 0x1A, '\n'};
    std::vector<uint8_t> ihdr;
    put32(ihdr, width);
    put32(ihdr, height);
    ihdr.insert(ihdr.end(), {8, uint8_t(rgb ? 2 : 6), 0, 0, 0});  // depth 8, colour type, deflate, filter 0, no interlace
    chunk(png, "IHDR", ihdr);
    chunk(png, "IDAT", z);
    chunk(png, "IEND", {});
    return png;
}

void write_file(const std::string& path, std::span<const uint8_t> data)
{
    std::ofstream f(path, std::ios::binary);
    f.write(reinterpret_cast<const char*>(data.data()), std::streamsize(data.size()));
    if (!f)
        throw std::runtime_error("cannot write " + path);
}

std::vector<uint8_t> with_provenance(std::vector<uint8_t> png, const Provenance& p)
{
    // IEND is the last 12 bytes (length 0, type, CRC); the text chunks go in front of it.
    if (png.size() < 20 || std::memcmp(png.data() + png.size() - 8, "IEND", 4) != 0)
        throw std::runtime_error("with_provenance: not a PNG ending in IEND");
    const char* sampler = p.sampler == "euler_a" ? "Euler a" : p.sampler == "er_sde" ? "ER-SDE" : "Euler";
    std::string params = p.prompt;
    if (p.negative)
        params += "\nNegative prompt: " + *p.negative;
    params += "\nSteps: " + std::to_string(p.steps) + ", Sampler: " + sampler + ", CFG scale: " + num_g(p.guidance) +
              ", Seed: " + std::to_string(p.seed) + ", Size: " + std::to_string(p.width) + "x" +
              std::to_string(p.height) + ", Model: " + p.model;
    std::string loras;
    for (const auto& l : p.loras)
        loras += (loras.empty() ? "" : ",") + std::string("{\"name\":") + json_string(l.name) +
                 ",\"scale\":" + num_g(l.scale) + "}";
    if (!p.loras.empty()) {
        params += ", Lora: ";
        for (size_t i = 0; i < p.loras.size(); ++i)
            params += (i ? " " : "") + p.loras[i].name + ":" + num_g(p.loras[i].scale);
    }
    const std::string json = "{\"prompt\":" + json_string(p.prompt) + ",\"negative_prompt\":" +
                             (p.negative ? json_string(*p.negative) : "null") + ",\"model\":" + json_string(p.model) +
                             ",\"steps\":" + std::to_string(p.steps) + ",\"guidance\":" + num_g(p.guidance) +
                             ",\"sampler\":" + json_string(p.sampler) + ",\"seed\":" + std::to_string(p.seed) +
                             ",\"width\":" + std::to_string(p.width) + ",\"height\":" + std::to_string(p.height) +
                             ",\"loras\":[" + loras + "]}";
    std::vector<uint8_t> chunks = itxt("parameters", params);
    const auto m = itxt("mako", json);
    chunks.insert(chunks.end(), m.begin(), m.end());
    png.insert(png.end() - 12, chunks.begin(), chunks.end());
    return png;
}

}  // namespace mkb::image

extern "C" {

mkb_status mkb_to_rgba8(const float* rgba, size_t count, uint8_t* out)
{
    if ((!rgba || !out) && count)
        return mkb::fail(MKB_ERR_INVALID, "to_rgba8: null argument");
    const auto v = mkb::image::to_rgba8(std::span<const float>(rgba, count));
    if (count)
        std::memcpy(out, v.data(), count);
    return MKB_OK;
}

mkb_status mkb_png_encode(const uint8_t* rgba8, uint32_t width, uint32_t height, int rgb, uint8_t* out,
                          size_t capacity, size_t* size)
{
    if (!rgba8 || !size)
        return mkb::fail(MKB_ERR_INVALID, "png_encode: null argument");
    try {
        const auto png =
            mkb::image::encode_png(std::span<const uint8_t>(rgba8, size_t(width) * height * 4), width, height, rgb);
        *size = png.size();
        if (!out)
            return MKB_OK;
        if (capacity < png.size())
            return mkb::fail(MKB_ERR_INVALID, "png_encode: output buffer too small");
        std::memcpy(out, png.data(), png.size());
        return MKB_OK;
    } catch (const std::exception& e) {
        return mkb::fail(MKB_ERR_INVALID, e.what());
    }
}

}  // extern "C"
