// A minimal safetensors reader: the header (an 8-byte little-endian length, then a JSON object of
// name -> {dtype, shape, data_offsets}) is parsed once; tensor data is read on demand with pread and converted to
// fp32. This is the checkpoint format the reference loads its transformer and LoRA files from
// (src/image/qwen_image.cpp:79-111 via its safetensors::Files).
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace mkb::st {

enum class DType { F32, F16, BF16, Other };

struct Tensor {
    std::string name;
    std::string dtype_name;  // as written in the header ("F32", "BF16", ...)
    DType dtype = DType::Other;
    std::vector<int64_t> shape;
    uint64_t begin = 0, end = 0;  // byte range within the data section
    int64_t count() const
    {
        int64_t n = 1;
        for (int64_t d : shape)
            n *= d;
        return n;
    }
};

class File {
public:
    // Opens and parses the header; null with *err set on any malformed input.
    static std::unique_ptr<File> open(const std::string& path, std::string* err);
    ~File();
    File(const File&) = delete;
    File& operator=(const File&) = delete;

    const std::vector<Tensor>& tensors() const { return tensors_; }
    const Tensor* find(const std::string& name) const;
    const std::map<std::string, std::string>& metadata() const { return metadata_; }
    const std::string& path() const { return path_; }

    // The tensor's values as fp32 into out[count()]; false with *err on read errors or unsupported dtypes.
    bool read_f32(const Tensor& t, float* out, std::string* err) const;

private:
    File() = default;
    std::string path_;
    int fd_ = -1;
    uint64_t data_offset_ = 0, data_size_ = 0;
    std::vector<Tensor> tensors_;
    std::map<std::string, size_t> index_;
    std::map<std::string, std::string> metadata_;
};

// IEEE binary16 -> binary32 (exact).
float half_to_float(uint16_t h);

}  // namespace mkb::st
