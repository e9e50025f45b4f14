// LoRA adapter files: pairs of <module>.lora_A / lora_B (or lora_down / lora_up) .weight tensors with an optional
// scalar <module>.alpha, handed one module at a time to a model's merge.
#pragma once

#include "mkb_image.h"

#include <functional>
#include <string>

namespace mkb {

// merge(module, A [rank][in], B [out][rank], rank, in, out, scale): scale includes alpha / rank when alpha is given.
using LoraMerge = std::function<mkb_status(const std::string&, const float*, const float*, int, int, int, float)>;

// Reads every pair of the file at `path` (file prefixes "transformer.", "diffusion_model.", "base_model.model.",
// "lora_unet_" dropped) and merges them; *merged (optional) counts the modules.
mkb_status load_lora_file(const char* path, float scale, const LoraMerge& merge, int* merged);

}  // namespace mkb
