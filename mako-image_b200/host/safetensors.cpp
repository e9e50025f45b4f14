#include "safetensors.hpp"

#include <cerrno>
#include <cstring>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

namespace mkb::st {

namespace {

// JSON values of the header: objects, arrays, strings, integers (and the literals, which are skipped).
struct Json {
    enum Kind { kNull, kBool, kNumber, kString, kArray, kObject } kind = kNull;
    std::string str;
    int64_t num = 0;
    bool num_is_int = true;
    std::vector<Json> items;                             // array
    std::vector<std::pair<std::string, Json>> members;  // object, in file order
};

class Parser {
public:
    Parser(const char* p, size_t n) : p_(p), end_(p + n) {}
    bool parse(Json& out, std::string* err)
    {
        if (!value(out, 0)) {
            *err = "safetensors: malformed header JSON (" + why_ + ")";
            return false;
        }
        ws();
        if (p_ != end_) {
            *err = "safetensors: trailing bytes after the header JSON";
            return false;
        }
        return true;
    }

private:
    const char* p_;
    const char* end_;
    std::string why_;

    bool fail(const char* w)
    {
        why_ = w;
        return false;
    }
    void ws()
    {
        while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r'))
            ++p_;
    }
    bool literal(const char* lit)
    {
        const size_t n = std::strlen(lit);
        if (size_t(end_ - p_) < n || std::memcmp(p_, lit, n) != 0)
            return fail("bad literal");
        p_ += n;
        return true;
    }
    static void put_utf8(std::string& s, uint32_t c)
    {
        if (c < 0x80) {
            s += char(c);
        } else if (c < 0x800) {
            s += char(0xC0 | (c >> 6));
            s += char(0x80 | (c & 0x3F));
        } else if (c < 0x10000) {
            s += char(0xE0 | (c >> 12));
            s += char(0x80 | ((c >> 6) & 0x3F));
            s += char(0x80 | (c & 0x3F));
        } else {
            s += char(0xF0 | (c >> 18));
            s += char(0x80 | ((c >> 12) & 0x3F));
            s += char(0x80 | ((c >> 6) & 0x3F));
            s += char(0x80 | (c & 0x3F));
        }
    }
    bool hex4(uint32_t& v)
    {
        if (end_ - p_ < 4)
            return fail("short \\u escape");
        v = 0;
        for (int i = 0; i < 4; ++i) {
            const char c = *p_++;
            v <<= 4;
            if (c >= '0' && c <= '9')
                v |= uint32_t(c - '0');
            else if (c >= 'a' && c <= 'f')
                v |= uint32_t(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F')
                v |= uint32_t(c - 'A' + 10);
            else
                return fail("bad \\u escape");
        }
        return true;
    }
    bool string(std::string& s)
    {
        if (p_ >= end_ || *p_ != '"')
            return fail("expected a string");
        ++p_;
        while (true) {
            if (p_ >= end_)
                return fail("unterminated string");
            const char c = *p_++;
            if (c == '"')
                return true;
            if (c != '\\') {
                s += c;
                continue;
            }
            if (p_ >= end_)
                return fail("unterminated escape");
            const char e = *p_++;
            switch (e) {
            case '"': s += '"'; break;
            case '\\': s += '\\'; break;
            case '/': s += '/'; break;
            case 'b': s += '\b'; break;
            case 'f': s += '\f'; break;
            case 'n': s += '\n'; break;
            case 'r': s += '\r'; break;
            case 't': s += '\t'; break;
            case 'u': {
                uint32_t c1 = 0;
                if (!hex4(c1))
                    return false;
                if (c1 >= 0xD800 && c1 < 0xDC00) {  // surrogate pair
                    uint32_t c2 = 0;
                    if (end_ - p_ < 2 || p_[0] != '\\' || p_[1] != 'u')
                        return fail("lone surrogate");
                    p_ += 2;
                    if (!hex4(c2) || c2 < 0xDC00 || c2 >= 0xE000)
                        return fail("bad surrogate pair");
                    c1 = 0x10000 + ((c1 - 0xD800) << 10) + (c2 - 0xDC00);
                }
                put_utf8(s, c1);
                break;
            }
            default: return fail("bad escape");
            }
        }
    }
    bool number(Json& v)
    {
        const char* s = p_;
        if (p_ < end_ && (*p_ == '-' || *p_ == '+'))
            ++p_;
        bool any = false, is_int = true;
        while (p_ < end_ && ((*p_ >= '0' && *p_ <= '9') || *p_ == '.' || *p_ == 'e' || *p_ == 'E' ||
                             ((*p_ == '-' || *p_ == '+') && (p_[-1] == 'e' || p_[-1] == 'E')))) {
            if (*p_ < '0' || *p_ > '9')
                is_int = false;
            any = true;
            ++p_;
        }
        if (!any)
            return fail("bad number");
        v.kind = Json::kNumber;
        v.num_is_int = is_int;
        if (is_int) {
            errno = 0;
            char* e = nullptr;
            const long long x = std::strtoll(std::string(s, p_).c_str(), &e, 10);
            if (errno)
                return fail("integer out of range");
            v.num = x;
        }
        return true;
    }
    bool value(Json& v, int depth)
    {
        if (depth > 64)
            return fail("nesting too deep");
        ws();
        if (p_ >= end_)
            return fail("unexpected end");
        const char c = *p_;
        if (c == '{') {
            ++p_;
            v.kind = Json::kObject;
            ws();
            if (p_ < end_ && *p_ == '}') {
                ++p_;
                return true;
            }
            while (true) {
                ws();
                std::string key;
                if (!string(key))
                    return false;
                ws();
                if (p_ >= end_ || *p_ != ':')
                    return fail("expected ':'");
                ++p_;
                Json child;
                if (!value(child, depth + 1))
                    return false;
                v.members.emplace_back(std::move(key), std::move(child));
                ws();
                if (p_ < end_ && *p_ == ',') {
                    ++p_;
                    continue;
                }
                if (p_ < end_ && *p_ == '}') {
                    ++p_;
                    return true;
                }
                return fail("expected ',' or '}'");
            }
        }
        if (c == '[') {
            ++p_;
            v.kind = Json::kArray;
            ws();
            if (p_ < end_ && *p_ == ']') {
                ++p_;
                return true;
            }
            while (true) {
                Json child;
                if (!value(child, depth + 1))
                    return false;
                v.items.push_back(std::move(child));
                ws();
                if (p_ < end_ && *p_ == ',') {
                    ++p_;
                    continue;
                }
                if (p_ < end_ && *p_ == ']') {
                    ++p_;
                    return true;
                }
                return fail("expected ',' or ']'");
            }
        }
        if (c == '"') {
            v.kind = Json::kString;
            return string(v.str);
        }
        if (c == 't' || c == 'f') {
            v.kind = Json::kBool;
            return literal(c == 't' ? "true" : "false");
        }
        if (c == 'n')
            return literal("null");
        return number(v);
    }
};

size_t dtype_size(DType d) { return d == DType::F32 ? 4 : 2; }

}  // namespace

float half_to_float(uint16_t h)
{
    const uint32_t sign = uint32_t(h & 0x8000) << 16;
    uint32_t exp = (h >> 10) & 0x1F, man = h & 0x3FF, bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;  // +-0
        } else {          // subnormal: normalise the mantissa
            int e = -1;
            do {
                ++e;
                man <<= 1;
            } while (!(man & 0x400));
            bits = sign | (uint32_t(127 - 15 - e) << 23) | ((man & 0x3FF) << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (man << 13);  // inf / nan
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

File::~File()
{
    if (fd_ >= 0)
        ::close(fd_);
}

std::unique_ptr<File> File::open(const std::string& path, std::string* err)
{
    std::unique_ptr<File> f(new File());
    f->path_ = path;
    f->fd_ = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (f->fd_ < 0) {
        *err = "safetensors: cannot open " + path + ": " + std::strerror(errno);
        return nullptr;
    }
    struct stat sb;
    if (fstat(f->fd_, &sb) != 0) {
        *err = "safetensors: cannot stat " + path;
        return nullptr;
    }
    const uint64_t fsize = uint64_t(sb.st_size);
    uint8_t lenb[8];
    if (fsize < 8 || pread(f->fd_, lenb, 8, 0) != 8) {
        *err = "safetensors: " + path + " is shorter than its header length";
        return nullptr;
    }
    uint64_t hlen = 0;
    for (int i = 7; i >= 0; --i)
        hlen = (hlen << 8) | lenb[i];
    if (hlen == 0 || hlen > (uint64_t(100) << 20) || 8 + hlen > fsize) {
        *err = "safetensors: " + path + " has a bad header length";
        return nullptr;
    }
    std::string hdr(hlen, '\0');
    if (pread(f->fd_, hdr.data(), hlen, 8) != ssize_t(hlen)) {
        *err = "safetensors: short read of the header of " + path;
        return nullptr;
    }
    Json root;
    if (!Parser(hdr.data(), hdr.size()).parse(root, err))
        return nullptr;
    if (root.kind != Json::kObject) {
        *err = "safetensors: the header is not a JSON object";
        return nullptr;
    }
    f->data_offset_ = 8 + hlen;
    f->data_size_ = fsize - f->data_offset_;
    for (auto& [name, v] : root.members) {
        if (name == "__metadata__") {
            if (v.kind == Json::kObject)
                for (auto& [k, mv] : v.members)
                    if (mv.kind == Json::kString)
                        f->metadata_[k] = mv.str;
            continue;
        }
        if (v.kind != Json::kObject) {
            *err = "safetensors: entry " + name + " is not an object";
            return nullptr;
        }
        Tensor t;
        t.name = name;
        const Json *dt = nullptr, *shape = nullptr, *offs = nullptr;
        for (auto& [k, mv] : v.members) {
            if (k == "dtype")
                dt = &mv;
            else if (k == "shape")
                shape = &mv;
            else if (k == "data_offsets")
                offs = &mv;
        }
        if (!dt || dt->kind != Json::kString || !shape || shape->kind != Json::kArray || !offs ||
            offs->kind != Json::kArray || offs->items.size() != 2) {
            *err = "safetensors: entry " + name + " lacks dtype, shape or data_offsets";
            return nullptr;
        }
        t.dtype_name = dt->str;
        t.dtype = dt->str == "F32" ? DType::F32 : dt->str == "F16" ? DType::F16 : dt->str == "BF16" ? DType::BF16
                                                                                                    : DType::Other;
        // The element count is checked as it is formed: a header whose dimensions overflow 64 bits (or exceed 2^48
        // elements, far beyond any checkpoint) could otherwise wrap around to a product that matches its byte range.
        int64_t elems = 1;
        for (const Json& d : shape->items) {
            if (d.kind != Json::kNumber || !d.num_is_int || d.num < 0) {
                *err = "safetensors: entry " + name + " has a bad shape";
                return nullptr;
            }
            if (__builtin_mul_overflow(elems, int64_t(d.num), &elems) || elems > (int64_t(1) << 48)) {
                *err = "safetensors: entry " + name + " has a shape too large to address";
                return nullptr;
            }
            t.shape.push_back(d.num);
        }
        for (const Json& o : offs->items)
            if (o.kind != Json::kNumber || !o.num_is_int || o.num < 0) {
                *err = "safetensors: entry " + name + " has bad data offsets";
                return nullptr;
            }
        t.begin = uint64_t(offs->items[0].num);
        t.end = uint64_t(offs->items[1].num);
        if (t.end < t.begin || t.end > f->data_size_) {
            *err = "safetensors: entry " + name + " lies outside the file";
            return nullptr;
        }
        if (t.dtype != DType::Other && uint64_t(t.count()) * dtype_size(t.dtype) != t.end - t.begin) {
            *err = "safetensors: entry " + name + " has a size that does not match its shape and dtype";
            return nullptr;
        }
        if (f->index_.count(name)) {
            *err = "safetensors: duplicate entry " + name;
            return nullptr;
        }
        f->index_[name] = f->tensors_.size();
        f->tensors_.push_back(std::move(t));
    }
    return f;
}

const Tensor* File::find(const std::string& name) const
{
    auto it = index_.find(name);
    return it == index_.end() ? nullptr : &tensors_[it->second];
}

bool File::read_f32(const Tensor& t, float* out, std::string* err) const
{
    if (t.dtype == DType::Other) {
        *err = "safetensors: " + t.name + " has unsupported dtype " + t.dtype_name + " (F32, F16 or BF16 only)";
        return false;
    }
    const uint64_t bytes = t.end - t.begin, n = uint64_t(t.count());
    std::vector<uint8_t> raw(bytes);
    uint64_t done = 0;
    while (done < bytes) {
        const ssize_t r = pread(fd_, raw.data() + done, bytes - done, off_t(data_offset_ + t.begin + done));
        if (r <= 0) {
            *err = "safetensors: short read of " + t.name + " in " + path_;
            return false;
        }
        done += uint64_t(r);
    }
    if (t.dtype == DType::F32) {
        std::memcpy(out, raw.data(), n * 4);
    } else {
        for (uint64_t i = 0; i < n; ++i) {
            const uint16_t h = uint16_t(raw[2 * i] | (raw[2 * i + 1] << 8));
            if (t.dtype == DType::F16) {
                out[i] = half_to_float(h);
            } else {
                const uint32_t b = uint32_t(h) << 16;
                std::memcpy(out + i, &b, 4);
            }
        }
    }
    return true;
}

}  // namespace mkb::st
