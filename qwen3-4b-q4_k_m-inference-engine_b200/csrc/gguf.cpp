// GGUF reader (gguf.h): the file is mapped read-only and parsed with a
// bounds-checked cursor, so a truncated or corrupt file is an error, never
// an out-of-range read.
#include "gguf.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>

#include "engine.h"

namespace q4k {
namespace {

constexpr uint32_t kMagic = 0x46554747u;  // "GGUF" read as a little-endian u32

enum : uint32_t {
    kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32 = 6, kBool = 7,
    kString = 8, kArray = 9, kU64 = 10, kI64 = 11, kF64 = 12,
};

[[noreturn]] void bad(const std::string& what) { throw Error(Q4K_EINVAL, "GGUF: " + what); }

class Cursor {
public:
    Cursor(const uint8_t* p, size_t n) : p_(p), n_(n) {}
    size_t pos() const { return at_; }
    template <class T>
    T get() {
        need(sizeof(T));
        T v;
        std::memcpy(&v, p_ + at_, sizeof(T));
        at_ += sizeof(T);
        return v;
    }
    std::string str() {
        const uint64_t len = get<uint64_t>();
        need(len);
        std::string s(reinterpret_cast<const char*>(p_ + at_), (size_t)len);
        at_ += (size_t)len;
        return s;
    }
    void skip(uint64_t bytes) {
        need(bytes);
        at_ += (size_t)bytes;
    }

private:
    void need(uint64_t bytes) const {
        if (bytes > n_ - at_) bad("truncated file");
    }
    const uint8_t* p_;
    size_t n_;
    size_t at_ = 0;
};

uint64_t scalar_size(uint32_t type) {
    switch (type) {
        case kU8: case kI8: case kBool: return 1;
        case kU16: case kI16: return 2;
        case kU32: case kI32: case kF32: return 4;
        case kU64: case kI64: case kF64: return 8;
        default: return 0;
    }
}

void skip_value(Cursor& c, uint32_t type, int depth) {
    if (depth > 4) bad("arrays nested too deeply");
    if (type == kString) {
        c.str();
    } else if (type == kArray) {
        const uint32_t et = c.get<uint32_t>();
        const uint64_t n = c.get<uint64_t>();
        const uint64_t sz = scalar_size(et);
        if (sz) {
            if (n > (uint64_t)1 << 40) bad("array too long");
            c.skip(n * sz);
        } else {
            for (uint64_t k = 0; k < n; ++k) skip_value(c, et, depth + 1);
        }
    } else {
        const uint64_t sz = scalar_size(type);
        if (!sz) bad("unknown value type " + std::to_string(type));
        c.skip(sz);
    }
}

GgufValue read_value(Cursor& c, uint32_t type) {
    GgufValue v;
    switch (type) {
        case kU8: v.kind = GgufValue::kUInt; v.u = c.get<uint8_t>(); break;
        case kU16: v.kind = GgufValue::kUInt; v.u = c.get<uint16_t>(); break;
        case kU32: v.kind = GgufValue::kUInt; v.u = c.get<uint32_t>(); break;
        case kU64: v.kind = GgufValue::kUInt; v.u = c.get<uint64_t>(); break;
        case kI8: v.kind = GgufValue::kInt; v.i = c.get<int8_t>(); break;
        case kI16: v.kind = GgufValue::kInt; v.i = c.get<int16_t>(); break;
        case kI32: v.kind = GgufValue::kInt; v.i = c.get<int32_t>(); break;
        case kI64: v.kind = GgufValue::kInt; v.i = c.get<int64_t>(); break;
        case kF32: v.kind = GgufValue::kFloat; v.f = c.get<float>(); break;
        case kF64: v.kind = GgufValue::kFloat; v.f = c.get<double>(); break;
        case kBool: v.kind = GgufValue::kBool; v.u = c.get<uint8_t>() != 0; break;
        case kString: v.kind = GgufValue::kString; v.s = c.str(); break;
        case kArray: {
            v.kind = GgufValue::kArray;
            v.array_type = c.get<uint32_t>();
            v.array_count = c.get<uint64_t>();
            const uint64_t sz = scalar_size(v.array_type);
            if (sz) {
                if (v.array_count > (uint64_t)1 << 40) bad("array too long");
                c.skip(v.array_count * sz);
            } else {
                for (uint64_t k = 0; k < v.array_count; ++k) skip_value(c, v.array_type, 1);
            }
            break;
        }
        default: bad("unknown value type " + std::to_string(type));
    }
    return v;
}

}  // namespace

bool GgufValue::as_int(int64_t& out) const {
    if (kind == kInt) {
        out = i;
        return true;
    }
    if (kind == kUInt && u <= (uint64_t)INT64_MAX) {
        out = (int64_t)u;
        return true;
    }
    return false;
}

bool GgufValue::as_float(double& out) const {
    int64_t n;
    if (kind == kFloat) {
        out = f;
        return true;
    }
    if (as_int(n)) {
        out = (double)n;
        return true;
    }
    return false;
}

uint64_t gguf_tensor_bytes(uint32_t type, int64_t ne0, int64_t rows) {
    if (ne0 <= 0 || rows <= 0) return 0;
    const uint64_t n = (uint64_t)ne0 * (uint64_t)rows;
    switch (type) {
        case 0: return 4 * n;  // F32
        case 1: return 2 * n;  // F16
        case 12: return ne0 % 256 ? 0 : n / 256 * 144;  // Q4_K
        case 14: return ne0 % 256 ? 0 : n / 256 * 210;  // Q6_K
        default: return 0;
    }
}

GgufFile::GgufFile(const std::string& path) {
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) throw Error(Q4K_EINVAL, "GGUF: cannot open " + path);
    struct stat st {};
    if (::fstat(fd, &st) != 0 || st.st_size < 24) {
        ::close(fd);
        bad(path + " is too short");
    }
    size_ = (size_t)st.st_size;
    void* m = ::mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (m == MAP_FAILED) throw Error(Q4K_EINVAL, "GGUF: cannot map " + path);
    base_ = static_cast<const uint8_t*>(m);
    try {
        Cursor c(base_, size_);
        if (c.get<uint32_t>() != kMagic) bad(path + " does not start with the GGUF magic");
        version_ = c.get<uint32_t>();
        if (version_ != 2 && version_ != 3) bad("unsupported version " + std::to_string(version_));
        const uint64_t n_tensors = c.get<uint64_t>(), n_kv = c.get<uint64_t>();
        if (n_tensors > (1u << 20) || n_kv > (1u << 20)) bad("implausible table sizes");
        for (uint64_t k = 0; k < n_kv; ++k) {
            std::string key = c.str();
            const uint32_t type = c.get<uint32_t>();
            meta_[key] = read_value(c, type);
        }
        tensors_.reserve((size_t)n_tensors);
        for (uint64_t k = 0; k < n_tensors; ++k) {
            GgufTensor t;
            t.name = c.str();
            const uint32_t nd = c.get<uint32_t>();
            if (nd == 0 || nd > 8) bad("tensor " + t.name + " has " + std::to_string(nd) + " dimensions");
            for (uint32_t d = 0; d < nd; ++d) {
                const uint64_t e = c.get<uint64_t>();
                if (e == 0 || e > ((uint64_t)1 << 40)) bad("tensor " + t.name + " has an invalid extent");
                t.ne.push_back((int64_t)e);
            }
            t.type = c.get<uint32_t>();
            t.offset = c.get<uint64_t>();
            int64_t rows = 1;
            for (size_t d = 1; d < t.ne.size(); ++d) rows *= t.ne[d];
            t.bytes = gguf_tensor_bytes(t.type, t.ne[0], rows);
            tensors_.push_back(std::move(t));
        }
        uint64_t align = 32;
        if (const GgufValue* a = find("general.alignment")) {
            int64_t v = 0;
            if (!a->as_int(v) || v <= 0 || (v & (v - 1))) bad("general.alignment must be a power of two");
            align = (uint64_t)v;
        }
        data_start_ = (c.pos() + align - 1) / align * align;
        for (const GgufTensor& t : tensors_) {
            if (t.offset % align) bad("tensor " + t.name + " is not aligned");
            if (data_start_ > size_ || t.offset > size_ - data_start_ || t.bytes > size_ - data_start_ - t.offset)
                bad("tensor " + t.name + " runs past the end of the file");
        }
    } catch (...) {
        ::munmap(const_cast<uint8_t*>(base_), size_);
        base_ = nullptr;
        throw;
    }
}

GgufFile::~GgufFile() {
    if (base_) ::munmap(const_cast<uint8_t*>(base_), size_);
}

const GgufValue* GgufFile::find(const std::string& key) const {
    auto it = meta_.find(key);
    return it == meta_.end() ? nullptr : &it->second;
}

const GgufTensor* GgufFile::tensor(const std::string& name) const {
    for (const GgufTensor& t : tensors_)
        if (t.name == name) return &t;
    return nullptr;
}

}  // namespace q4k
