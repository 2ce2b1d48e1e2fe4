// GGUF v2/v3 reader over a read-only mmap (host side).
//
// Restates the behaviour of smallm-engine's loader (src/core/gguf.cpp
// :116-183): magic check, typed metadata, tensor table, tensor data aligned
// to general.alignment (uint32, default 32), zero-copy views into the
// mapping; and its config readers (src/config/common/config.cpp:23-48,
// include/smallm/config/common/meta_read.h:14-34): required keys must exist
// with exactly the requested type, optional ones fall back.
#pragma once

#include <stdint.h>

#include <string>
#include <unordered_map>
#include <vector>

namespace smallm {

struct GGUFTensor {
    std::string name;
    std::vector<uint64_t> dims;  // fastest-moving first
    uint32_t type = 0;
    uint64_t offset = 0;         // relative to the data section
    uint64_t numel() const {
        uint64_t n = 1;
        for (uint64_t d : dims) n *= d;
        return n;
    }
};

struct GGUFMeta {
    uint32_t type = 0;             // GGUF value type id
    uint64_t raw = 0;              // scalar payload (little-endian bits)
    std::string str;               // STRING value
    uint32_t arr_type = 0;         // ARRAY element type
    uint64_t arr_len = 0;          // ARRAY length
};

class GGUFFile {
public:
    explicit GGUFFile(const std::string& path);
    ~GGUFFile();
    GGUFFile(const GGUFFile&) = delete;
    GGUFFile& operator=(const GGUFFile&) = delete;

    const GGUFTensor* find(const std::string& name) const;
    const GGUFTensor& tensor(const std::string& name) const;  // throws "tensor not found: <name>"
    const uint8_t* data(const GGUFTensor& t) const { return map_ + data_offset_ + t.offset; }

    // meta::get<T> (throws "config: missing metadata key" / "wrong type") and get_or
    uint32_t get_u32(const std::string& key) const;
    uint32_t get_u32_or(const std::string& key, uint32_t fallback) const;
    float get_f32_or(const std::string& key, float fallback) const;
    std::string get_str(const std::string& key) const;
    // length of a string array (0 if absent or not a string array)
    uint64_t str_array_len(const std::string& key) const;

    uint32_t version() const { return version_; }
    size_t size() const { return size_; }
    const uint8_t* mapping() const { return map_; }

private:
    const uint8_t* map_ = nullptr;
    size_t size_ = 0;
    uint64_t data_offset_ = 0;
    uint32_t version_ = 0;
    std::unordered_map<std::string, GGUFMeta> meta_;
    std::vector<GGUFTensor> tensors_;
    std::unordered_map<std::string, size_t> index_;
};

}  // namespace smallm
