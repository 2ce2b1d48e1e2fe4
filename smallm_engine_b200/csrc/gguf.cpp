#include "gguf.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>

#include "engine.h"

namespace smallm {

namespace {

enum : uint32_t {
    G_U8 = 0, G_I8 = 1, G_U16 = 2, G_I16 = 3, G_U32 = 4, G_I32 = 5, G_F32 = 6, G_BOOL = 7,
    G_STR = 8, G_ARR = 9, G_U64 = 10, G_I64 = 11, G_F64 = 12
};

struct Cursor {
    const uint8_t* base;
    size_t size;
    size_t pos = 0;
    void raw(void* out, size_t n) {
        if (pos + n > size || pos + n < pos) throw Error(5, "gguf: read past end of file");
        std::memcpy(out, base + pos, n);
        pos += n;
    }
    template <typename T>
    T get() {
        T v;
        raw(&v, sizeof(T));
        return v;
    }
    std::string str() {
        uint64_t n = get<uint64_t>();
        if (n > size - pos) throw Error(5, "gguf: string past end of file");
        std::string s(reinterpret_cast<const char*>(base + pos), n);
        pos += n;
        return s;
    }
    void skip(size_t n) {
        if (n > size - pos) throw Error(5, "gguf: read past end of file");
        pos += n;
    }
};

size_t scalar_size(uint32_t t) {
    switch (t) {
        case G_U8: case G_I8: case G_BOOL: return 1;
        case G_U16: case G_I16: return 2;
        case G_U32: case G_I32: case G_F32: return 4;
        case G_U64: case G_I64: case G_F64: return 8;
        default: return 0;
    }
}

GGUFMeta read_value(Cursor& c, uint32_t type) {
    GGUFMeta m;
    m.type = type;
    if (type == G_STR) {
        m.str = c.str();
    } else if (type == G_ARR) {
        m.arr_type = c.get<uint32_t>();
        m.arr_len = c.get<uint64_t>();
        if (m.arr_type == G_STR) {
            for (uint64_t i = 0; i < m.arr_len; ++i) c.skip(c.get<uint64_t>());
        } else {
            size_t es = scalar_size(m.arr_type);
            if (!es) throw Error(5, "gguf: unsupported array element type");
            if (m.arr_len > (c.size - c.pos) / es) throw Error(5, "gguf: read past end of file");
            c.skip(es * m.arr_len);
        }
    } else {
        size_t n = scalar_size(type);
        if (!n) throw Error(5, "gguf: unknown metadata value type");
        c.raw(&m.raw, n);
    }
    return m;
}

}  // namespace

GGUFFile::GGUFFile(const std::string& path) {
    int fd = open(path.c_str(), O_RDONLY);
    if (fd < 0) throw Error(4, "gguf: cannot open file: " + path);
    struct stat st {};
    if (fstat(fd, &st) != 0) {
        close(fd);
        throw Error(4, "gguf: fstat failed");
    }
    size_ = static_cast<size_t>(st.st_size);
    void* m = size_ ? mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0) : MAP_FAILED;
    close(fd);
    if (m == MAP_FAILED) throw Error(4, "gguf: mmap failed");
    map_ = static_cast<const uint8_t*>(m);
    try {
        Cursor c{map_, size_};
        char magic[4];
        c.raw(magic, 4);
        if (std::memcmp(magic, "GGUF", 4) != 0) throw Error(5, "gguf: bad magic, not a GGUF file");
        version_ = c.get<uint32_t>();
        const uint64_t nt = c.get<uint64_t>();
        const uint64_t nkv = c.get<uint64_t>();
        for (uint64_t i = 0; i < nkv; ++i) {
            std::string k = c.str();
            uint32_t t = c.get<uint32_t>();
            meta_[k] = read_value(c, t);
        }
        if (nt > size_) throw Error(5, "gguf: read past end of file");
        tensors_.reserve(nt);
        for (uint64_t i = 0; i < nt; ++i) {
            GGUFTensor t;
            t.name = c.str();
            uint32_t nd = c.get<uint32_t>();
            if (nd > 8) throw Error(5, "gguf: bad tensor rank");
            t.dims.resize(nd);
            for (uint32_t d = 0; d < nd; ++d) t.dims[d] = c.get<uint64_t>();
            t.type = c.get<uint32_t>();
            t.offset = c.get<uint64_t>();
            index_[t.name] = tensors_.size();
            tensors_.push_back(std::move(t));
        }
        uint32_t align = 32;
        auto it = meta_.find("general.alignment");
        if (it != meta_.end() && it->second.type == G_U32) align = (uint32_t)it->second.raw;
        if (align == 0) align = 32;
        data_offset_ = (c.pos + align - 1) / align * align;
        for (const auto& t : tensors_) {
            uint64_t rb = type_row_bytes(t.type, t.dims.empty() ? 1 : t.dims[0]);
            uint64_t rows = t.dims.empty() ? 1 : t.numel() / t.dims[0];
            if (type_supported(t.type) && data_offset_ + t.offset + rb * rows > size_)
                throw Error(5, "gguf: tensor " + t.name + " extends past end of file");
        }
    } catch (...) {
        munmap(const_cast<uint8_t*>(map_), size_);
        map_ = nullptr;
        throw;
    }
}

GGUFFile::~GGUFFile() {
    if (map_) munmap(const_cast<uint8_t*>(map_), size_);
}

const GGUFTensor* GGUFFile::find(const std::string& name) const {
    auto it = index_.find(name);
    return it == index_.end() ? nullptr : &tensors_[it->second];
}

const GGUFTensor& GGUFFile::tensor(const std::string& name) const {
    const GGUFTensor* t = find(name);
    if (!t) throw Error(5, "tensor not found: " + name);
    return *t;
}

uint32_t GGUFFile::get_u32(const std::string& key) const {
    auto it = meta_.find(key);
    if (it == meta_.end()) throw Error(5, "config: missing metadata key: " + key);
    if (it->second.type != G_U32) throw Error(5, "config: wrong type for metadata key: " + key);
    return (uint32_t)it->second.raw;
}

uint32_t GGUFFile::get_u32_or(const std::string& key, uint32_t fallback) const {
    auto it = meta_.find(key);
    if (it == meta_.end() || it->second.type != G_U32) return fallback;
    return (uint32_t)it->second.raw;
}

float GGUFFile::get_f32_or(const std::string& key, float fallback) const {
    auto it = meta_.find(key);
    if (it == meta_.end() || it->second.type != G_F32) return fallback;
    float f;
    uint32_t b = (uint32_t)it->second.raw;
    std::memcpy(&f, &b, 4);
    return f;
}

std::string GGUFFile::get_str(const std::string& key) const {
    auto it = meta_.find(key);
    if (it == meta_.end()) throw Error(5, "config: missing metadata key: " + key);
    if (it->second.type != G_STR) throw Error(5, "config: wrong type for metadata key: " + key);
    return it->second.str;
}

uint64_t GGUFFile::str_array_len(const std::string& key) const {
    auto it = meta_.find(key);
    if (it == meta_.end() || it->second.type != G_ARR || it->second.arr_type != G_STR) return 0;
    return it->second.arr_len;
}

}  // namespace smallm
