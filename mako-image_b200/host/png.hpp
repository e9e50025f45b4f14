// Image output for the drivers: 8-bit conversion and a PNG writer of this library's own (the reference writes PNGs
// through Apple's ImageIO, src/image/png.hpp:13-30, which does not exist here). Same names and meaning as the
// reference's to_rgba8 / encode_png / with_provenance / write_file; errors are std::runtime_error as there.
#pragma once

#include <cstdint>
#include <optional>
#include <span>
#include <string>
#include <vector>

namespace mkb::image {

// RGBA [height][width][4] in [-1, 1] to 8-bit samples: x / 2 + 1/2, clamped to [0, 1], times 255, rounded to
// nearest (ties to even), as the reference's pipeline makes them (png.cpp:148-156).
std::vector<uint8_t> to_rgba8(std::span<const float> rgba);

// A PNG of 8-bit RGBA [height][width][4] (colour type 6), or with `rgb` of its RGB samples (colour type 2, the alpha
// left out). The zlib stream holds stored deflate blocks (no compression: the encoder is a few dozen lines with no
// dependency, and a 1024^2 image is 4 MB).
std::vector<uint8_t> encode_png(std::span<const uint8_t> rgba8, uint32_t width, uint32_t height, bool rgb = false);

void write_file(const std::string& path, std::span<const uint8_t> data);

// How an image was made, for the PNG's text chunks (the reference's Provenance, png.hpp:33-55, with the fields this
// library's drivers fill).
struct Provenance {
    std::string prompt, model;
    std::optional<std::string> negative;  // when guided
    std::string sampler = "euler";        // "euler", "euler_a", "er_sde"
    float guidance = 1;
    uint32_t steps = 0, width = 0, height = 0;
    uint64_t seed = 0;
    struct Lora {
        std::string name;
        float scale = 1;
    };
    std::vector<Lora> loras;
};

// The PNG with two UTF-8 text chunks (iTXt) before its end: "parameters" (the prompt, then "Negative prompt: ...",
// then "Steps: ..., Sampler: ..., CFG scale: ..., Seed: ..., Size: WxH, Model: ...", the line image tools read) and
// "mako" (the same as JSON, with the LoRAs), as the reference's with_provenance (png.hpp:56-61) writes them.
// Throws std::runtime_error on data that is not a PNG.
std::vector<uint8_t> with_provenance(std::vector<uint8_t> png, const Provenance& p);

// CRC-32 (ISO 3309 / PNG) and Adler-32 (zlib), as the formats define them.
uint32_t crc32(std::span<const uint8_t> data, uint32_t crc = 0);
uint32_t adler32(std::span<const uint8_t> data, uint32_t adler = 1);

}  // namespace mkb::image
