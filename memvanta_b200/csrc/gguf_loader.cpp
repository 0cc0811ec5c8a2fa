// gguf_loader.cpp -- see gguf_loader.hpp.
#include "gguf_loader.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <limits>
#include <stdexcept>

namespace mvb {

namespace {

// Sequential little-endian cursor over the mapping with bounds checks.
class Cursor {
public:
    Cursor(const uint8_t* p, uint64_t n) : p_(p), n_(n) {}
    uint64_t pos() const { return at_; }
    void need(uint64_t k) const {
        if (k > n_ || at_ > n_ - k) throw std::runtime_error("truncated GGUF");
    }
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
        std::string s(reinterpret_cast<const char*>(p_ + at_), static_cast<size_t>(len));
        at_ += len;
        return s;
    }
    void skip(uint64_t k) {
        need(k);
        at_ += k;
    }

private:
    const uint8_t* p_;
    uint64_t n_;
    uint64_t at_ = 0;
};

// GGUF metadata value types.
enum : uint32_t { U8 = 0, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 };

uint64_t scalar_size(uint32_t t) {
    switch (t) {
        case U8: case I8: case BOOL: return 1;
        case U16: case I16: return 2;
        case U32: case I32: case F32: return 4;
        case U64: case I64: case F64: return 8;
    }
    return 0;
}

GgufValue read_scalar(Cursor& c, uint32_t t) {
    GgufValue v;
    switch (t) {
        case U8: v.kind = GgufValue::UInt; v.u = c.get<uint8_t>(); break;
        case U16: v.kind = GgufValue::UInt; v.u = c.get<uint16_t>(); break;
        case U32: v.kind = GgufValue::UInt; v.u = c.get<uint32_t>(); break;
        case U64: v.kind = GgufValue::UInt; v.u = c.get<uint64_t>(); break;
        case I8: v.kind = GgufValue::Int; v.i = c.get<int8_t>(); break;
        case I16: v.kind = GgufValue::Int; v.i = c.get<int16_t>(); break;
        case I32: v.kind = GgufValue::Int; v.i = c.get<int32_t>(); break;
        case I64: v.kind = GgufValue::Int; v.i = c.get<int64_t>(); break;
        case F32: v.kind = GgufValue::Float; v.f = c.get<float>(); break;
        case F64: v.kind = GgufValue::Float; v.f = c.get<double>(); break;
        case BOOL: v.kind = GgufValue::Bool; v.b = c.get<uint8_t>() != 0; break;
        case STR: v.kind = GgufValue::String; v.s = c.str(); break;
        default: throw std::runtime_error("unknown GGUF metadata type");
    }
    return v;
}

GgufValue read_value(Cursor& c, uint32_t t) {
    if (t != ARR) return read_scalar(c, t);
    const uint32_t et = c.get<uint32_t>();
    const uint64_t n = c.get<uint64_t>();
    GgufValue v;
    v.kind = GgufValue::Array;
    v.array_len = static_cast<size_t>(n);
    if (et == STR) {
        for (uint64_t i = 0; i < n; ++i) {
            const uint64_t len = c.get<uint64_t>();
            c.skip(len);
        }
    } else if (et == ARR) {
        throw std::runtime_error("nested GGUF arrays are unsupported");
    } else {
        const uint64_t sz = scalar_size(et);
        if (!sz) throw std::runtime_error("unknown GGUF array element type");
        if (n > std::numeric_limits<uint64_t>::max() / sz) throw std::runtime_error("GGUF array too large");
        c.skip(n * sz);
    }
    return v;
}

}  // namespace

uint64_t ggml_nbytes(uint32_t type, uint64_t n) {
    auto blocks = [&](uint64_t per, uint64_t bytes) {
        if (n % per) throw std::runtime_error("quantized tensor element count is not block aligned");
        return n / per * bytes;
    };
    switch (type) {
        case 0: return n * 4;     // F32
        case 1: return n * 2;     // F16
        case 2: return blocks(32, 18);   // Q4_0
        case 3: return blocks(32, 20);   // Q4_1
        case 6: return blocks(32, 22);   // Q5_0
        case 7: return blocks(32, 24);   // Q5_1
        case 8: return blocks(32, 34);   // Q8_0
        case 10: return blocks(256, 84);  // Q2_K
        case 11: return blocks(256, 110); // Q3_K
        case 12: return blocks(256, 144); // Q4_K
        case 13: return blocks(256, 176); // Q5_K
        case 14: return blocks(256, 210); // Q6_K
        case 24: return n;        // I8
        case 25: return n * 2;    // I16
        case 26: return n * 4;    // I32
        case 27: return n * 8;    // I64
        case 28: return n * 8;    // F64
        case 30: return n * 2;    // BF16
    }
    throw std::runtime_error("unsupported GGML type for byte-size calculation: " + std::to_string(type));
}

uint64_t GgufTensorInfo::elements() const {
    uint64_t n = 1;
    for (uint64_t d : dims) {
        if (d && n > std::numeric_limits<uint64_t>::max() / d) throw std::runtime_error("tensor element overflow");
        n *= d;
    }
    return n;
}

GgufReader::GgufReader(const std::string& path) {
    fd_ = ::open(path.c_str(), O_RDONLY);
    if (fd_ < 0) throw std::runtime_error("open failed: " + path);
    struct stat st {};
    if (fstat(fd_, &st) != 0 || st.st_size <= 0) {
        ::close(fd_);
        fd_ = -1;
        throw std::runtime_error("empty or unreadable file: " + path);
    }
    size_ = static_cast<uint64_t>(st.st_size);
    void* p = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
    if (p == MAP_FAILED) {
        ::close(fd_);
        fd_ = -1;
        throw std::runtime_error("mmap failed: " + path);
    }
    base_ = static_cast<uint8_t*>(p);
    try {
        Cursor c(base_, size_);
        if (c.get<uint32_t>() != 0x46554747u) throw std::runtime_error("not a GGUF file");  // "GGUF"
        version_ = c.get<uint32_t>();
        if (version_ < 2 || version_ > 3) throw std::runtime_error("unsupported GGUF version: " + std::to_string(version_));
        const uint64_t nt = c.get<uint64_t>(), nkv = c.get<uint64_t>();
        if (nt > 1000000 || nkv > 1000000) throw std::runtime_error("implausible GGUF counts");
        for (uint64_t i = 0; i < nkv; ++i) {
            std::string key = c.str();
            const uint32_t t = c.get<uint32_t>();
            meta_[key] = read_value(c, t);
        }
        struct Raw {
            GgufTensorInfo info;
            uint64_t rel;
        };
        std::vector<Raw> raw;
        raw.reserve(static_cast<size_t>(nt));
        for (uint64_t i = 0; i < nt; ++i) {
            Raw r;
            r.info.name = c.str();
            const uint32_t nd = c.get<uint32_t>();
            if (nd == 0 || nd > 4) throw std::runtime_error("invalid tensor dimensions");
            r.info.dims.resize(nd);
            for (auto& d : r.info.dims) d = c.get<uint64_t>();
            r.info.type = c.get<uint32_t>();
            r.rel = c.get<uint64_t>();
            raw.push_back(std::move(r));
        }
        uint64_t align = 32;
        uint64_t a;
        if (get_u64("general.alignment", a)) align = a;
        if (!align || (align & (align - 1))) throw std::runtime_error("invalid GGUF alignment");
        const uint64_t data_start = (c.pos() + align - 1) & ~(align - 1);
        // a huge alignment wraps the rounding
        if (data_start < c.pos()) throw std::runtime_error("invalid GGUF alignment");
        for (auto& r : raw) {
            // checked before the add: a relative offset near 2^64 would wrap
            if (data_start > size_ || r.rel > size_ - data_start)
                throw std::runtime_error("tensor out of file bounds: " + r.info.name);
            r.info.offset = data_start + r.rel;
            r.info.nbytes = ggml_nbytes(r.info.type, r.info.elements());
            if (r.info.offset > size_ || r.info.nbytes > size_ - r.info.offset)
                throw std::runtime_error("tensor out of file bounds: " + r.info.name);
            index_[r.info.name] = tensors_.size();
            tensors_.push_back(std::move(r.info));
        }
    } catch (...) {
        munmap(base_, size_);
        ::close(fd_);
        base_ = nullptr;
        fd_ = -1;
        throw;
    }
}

GgufReader::~GgufReader() {
    if (base_) munmap(base_, size_);
    if (fd_ >= 0) ::close(fd_);
}

const GgufTensorInfo* GgufReader::find(const std::string& name) const {
    auto it = index_.find(name);
    return it == index_.end() ? nullptr : &tensors_[it->second];
}

const GgufTensorInfo& GgufReader::tensor(const std::string& name) const {
    const GgufTensorInfo* t = find(name);
    if (!t) throw std::runtime_error("missing tensor: " + name);
    return *t;
}

bool GgufReader::get_u64(const std::string& key, uint64_t& out) const {
    auto it = meta_.find(key);
    if (it == meta_.end()) return false;
    if (it->second.kind == GgufValue::UInt) { out = it->second.u; return true; }
    if (it->second.kind == GgufValue::Int && it->second.i >= 0) { out = static_cast<uint64_t>(it->second.i); return true; }
    return false;
}

bool GgufReader::get_f64(const std::string& key, double& out) const {
    auto it = meta_.find(key);
    if (it == meta_.end()) return false;
    switch (it->second.kind) {
        case GgufValue::Float: out = it->second.f; return true;
        case GgufValue::UInt: out = static_cast<double>(it->second.u); return true;
        case GgufValue::Int: out = static_cast<double>(it->second.i); return true;
        default: return false;
    }
}

bool GgufReader::get_string(const std::string& key, std::string& out) const {
    auto it = meta_.find(key);
    if (it == meta_.end() || it->second.kind != GgufValue::String) return false;
    out = it->second.s;
    return true;
}

void GgufReader::advise_sequential() const {
    if (base_) madvise(base_, size_, MADV_SEQUENTIAL);
}

}  // namespace mvb
