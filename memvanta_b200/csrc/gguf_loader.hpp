// gguf_loader.hpp -- host-side GGUF reader for the device model.
//
// Same job as the reference's GgufFile (include/memvanta/gguf.hpp:72-111,
// src/gguf.cpp:121-139): mmap the file read-only, parse the v2/v3 header,
// the key/value metadata and the tensor table, align the data section and
// check every tensor lies inside the file.  The weights are not copied on the
// host: the model uploads each tensor's blocks from the mapping straight to
// HBM.
#pragma once
#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace mvb {

struct GgufTensorInfo {
    std::string name;
    std::vector<uint64_t> dims;  // ne0 (cols), ne1 (rows), ...
    uint32_t type = 0;
    uint64_t offset = 0;         // absolute file offset
    uint64_t nbytes = 0;
    uint64_t ne(size_t i) const { return i < dims.size() ? dims[i] : 1; }
    uint64_t elements() const;
};

struct GgufValue {
    enum Kind { UInt, Int, Float, Bool, String, Array } kind = UInt;
    uint64_t u = 0;
    int64_t i = 0;
    double f = 0.0;
    bool b = false;
    std::string s;
    size_t array_len = 0;  // arrays are skipped, only their length is kept
};

class GgufReader {
public:
    explicit GgufReader(const std::string& path);  // throws std::runtime_error
    ~GgufReader();
    GgufReader(const GgufReader&) = delete;
    GgufReader& operator=(const GgufReader&) = delete;

    uint32_t version() const { return version_; }
    const std::vector<GgufTensorInfo>& tensors() const { return tensors_; }
    const GgufTensorInfo* find(const std::string& name) const;
    const GgufTensorInfo& tensor(const std::string& name) const;  // throws "missing tensor: <name>"
    const uint8_t* data(const GgufTensorInfo& t) const { return base_ + t.offset; }

    bool has(const std::string& key) const { return meta_.count(key) != 0; }
    bool get_u64(const std::string& key, uint64_t& out) const;
    bool get_f64(const std::string& key, double& out) const;
    bool get_string(const std::string& key, std::string& out) const;
    void advise_sequential() const;

private:
    int fd_ = -1;
    uint8_t* base_ = nullptr;
    uint64_t size_ = 0;
    uint32_t version_ = 0;
    std::map<std::string, GgufValue> meta_;
    std::vector<GgufTensorInfo> tensors_;
    std::map<std::string, size_t> index_;
};

uint64_t ggml_nbytes(uint32_t type, uint64_t elements);  // throws on unknown types / misalignment

}  // namespace mvb
