// gguf.cpp -- GGUF reader (see gguf.hpp).
#include "gguf.hpp"

#include <errno.h>
#include <fcntl.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace ge {

namespace {
constexpr int kFileNotReadable = 1, kInvalidGguf = 2, kUnsupportedType = 3;

struct Cursor {
    const uint8_t* base;
    size_t size, pos;
    bool need(size_t n) const { return pos <= size && n <= size - pos; }
    template <class T>
    bool read(T& v) {
        if (!need(sizeof(T))) return false;
        memcpy(&v, base + pos, sizeof(T));
        pos += sizeof(T);
        return true;
    }
    bool str(std::string& s) {
        uint64_t n;
        if (!read(n) || !need(n)) return false;
        s.assign(reinterpret_cast<const char*>(base + pos), n);
        pos += n;
        return true;
    }
};

int64_t fixed_size(uint32_t t) {
    switch (t) {
    case 0: case 1: case 7: return 1;
    case 2: case 3: return 2;
    case 4: case 5: case 6: return 4;
    case 10: case 11: case 12: return 8;
    default: return -1;
    }
}

// Skips one value of type `t` (GGUFFile.swift:124-176); false if truncated or unknown.
bool skip(Cursor& c, uint32_t t, int depth, bool& unknown) {
    if (t == 8) {
        std::string s;
        return c.str(s);
    }
    if (t == 9) {
        uint32_t et;
        uint64_t n;
        if (depth > 3 || !c.read(et) || !c.read(n)) return false;
        const int64_t fs = fixed_size(et);
        if (fs > 0) {
            if (n > c.size || !c.need(n * uint64_t(fs))) return false;
            c.pos += n * uint64_t(fs);
            return true;
        }
        for (uint64_t i = 0; i < n; i++)
            if (!skip(c, et, depth + 1, unknown)) return false;
        return true;
    }
    const int64_t fs = fixed_size(t);
    if (fs < 0) {
        unknown = true;
        return false;
    }
    if (!c.need(size_t(fs))) return false;
    c.pos += size_t(fs);
    return true;
}
}  // namespace

int64_t ggml_block_elems(uint32_t type) { return type == GGML_Q8_0 ? 32 : 1; }
int64_t ggml_block_bytes(uint32_t type) {
    switch (type) {
    case GGML_F32: return 4;
    case GGML_F16: case GGML_BF16: return 2;
    case GGML_Q8_0: return 34;
    default: return -1;
    }
}

int64_t GgufTensor::elements() const {
    int64_t n = 1;
    for (int64_t s : shape) n *= s;
    return n;
}
int64_t GgufTensor::bytes() const { return elements() / ggml_block_elems(type) * ggml_block_bytes(type); }

GgufFile::~GgufFile() {
    if (base_) munmap(base_, mapped_);
}

int GgufFile::open(const std::string& path, GgufError& err) {
    auto fail = [&](int code, const std::string& msg) {
        err.code = code;
        err.message = msg;
        return code;
    };
    int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) return fail(kFileNotReadable, "cannot read " + path + ": " + strerror(errno));
    struct stat st;
    if (fstat(fd, &st) != 0) {
        int e = errno;
        ::close(fd);
        return fail(kFileNotReadable, "cannot read " + path + ": " + strerror(e));
    }
    if (st.st_size <= 0) {
        ::close(fd);
        return fail(kInvalidGguf, "invalid GGUF file: file is empty");
    }
    size = size_t(st.st_size);
    const size_t page = size_t(sysconf(_SC_PAGESIZE));
    mapped_ = (size + page - 1) / page * page;
    void* p = mmap(nullptr, mapped_, PROT_READ, MAP_SHARED, fd, 0);
    ::close(fd);
    if (p == MAP_FAILED) return fail(kFileNotReadable, "cannot read " + path + ": mmap failed");
    base_ = static_cast<uint8_t*>(p);

    Cursor c{base_, size, 0};
    auto truncated = [&]() { return fail(kInvalidGguf, "invalid GGUF file: truncated header at byte " + std::to_string(c.pos)); };
    uint32_t magic = 0;
    if (!c.read(magic)) return truncated();
    if (magic != 0x46554747u) {
        char buf[64];
        snprintf(buf, sizeof buf, "invalid GGUF file: bad magic 0x%x", magic);
        return fail(kInvalidGguf, buf);
    }
    if (!c.read(version)) return truncated();
    if (version != 2 && version != 3)
        return fail(kInvalidGguf, "invalid GGUF file: unsupported version " + std::to_string(version));
    uint64_t ntensors = 0, nkv = 0;
    if (!c.read(ntensors) || !c.read(nkv)) return truncated();
    if (nkv > size || ntensors > size) return truncated();
    for (uint64_t i = 0; i < nkv; i++) {
        std::string key;
        GgufValue v;
        if (!c.str(key) || !c.read(v.type)) return truncated();
        if (v.type > 12) return fail(kInvalidGguf, "invalid GGUF file: unknown metadata value type " + std::to_string(v.type));
        if (v.type == 9) {
            if (!c.need(12)) return truncated();
            memcpy(&v.elem, base_ + c.pos, 4);
            memcpy(&v.count, base_ + c.pos + 4, 8);
            v.raw = base_ + c.pos + 12;
        } else {
            v.raw = base_ + c.pos;
        }
        bool unknown = false;
        if (!skip(c, v.type, 0, unknown)) {
            if (unknown) return fail(kInvalidGguf, "invalid GGUF file: unknown metadata value type");
            return truncated();
        }
        metadata[key] = v;
    }
    tensors.reserve(ntensors);
    for (uint64_t i = 0; i < ntensors; i++) {
        GgufTensor t;
        uint32_t nd = 0;
        if (!c.str(t.name) || !c.read(nd)) return truncated();
        if (nd > 4)
            return fail(kInvalidGguf, "invalid GGUF file: tensor " + t.name + " has " + std::to_string(nd) + " dimensions");
        for (uint32_t d = 0; d < nd; d++) {
            uint64_t s;
            if (!c.read(s)) return truncated();
            t.shape.push_back(int64_t(s));
        }
        if (!c.read(t.type) || !c.read(t.offset)) return truncated();
        if (ggml_block_bytes(t.type) < 0)
            return fail(kUnsupportedType, "tensor " + t.name + " uses unsupported storage type " + std::to_string(t.type));
        index_[t.name] = tensors.size();
        tensors.push_back(std::move(t));
    }
    int64_t alignment = 32;
    int64_t a;
    if (get_int("general.alignment", a) && a > 0) alignment = a;
    const size_t data = (c.pos + size_t(alignment) - 1) / size_t(alignment) * size_t(alignment);
    for (auto& t : tensors) {
        for (int64_t s : t.shape)
            if (s <= 0 || s > int64_t(size) * 32)
                return fail(kInvalidGguf, "invalid GGUF file: tensor " + t.name + " extends past the end of the file");
        const uint64_t end = uint64_t(data) + t.offset + uint64_t(t.bytes());
        if (t.offset > size || end > size)
            return fail(kInvalidGguf, "invalid GGUF file: tensor " + t.name + " extends past the end of the file");
        t.data = base_ + data + t.offset;
    }
    return 0;
}

const GgufTensor* GgufFile::tensor(const std::string& name) const {
    auto it = index_.find(name);
    return it == index_.end() ? nullptr : &tensors[it->second];
}

bool GgufFile::get_int(const std::string& key, int64_t& out) const {
    auto it = metadata.find(key);
    if (it == metadata.end()) return false;
    const uint8_t* p = it->second.raw;
    switch (it->second.type) {
    case 0: out = *p; return true;
    case 1: out = int8_t(*p); return true;
    case 2: { uint16_t v; memcpy(&v, p, 2); out = v; return true; }
    case 3: { int16_t v; memcpy(&v, p, 2); out = v; return true; }
    case 4: { uint32_t v; memcpy(&v, p, 4); out = v; return true; }
    case 5: { int32_t v; memcpy(&v, p, 4); out = v; return true; }
    case 10: { uint64_t v; memcpy(&v, p, 8); out = int64_t(v); return true; }
    case 11: { int64_t v; memcpy(&v, p, 8); out = v; return true; }
    default: return false;
    }
}

bool GgufFile::get_float(const std::string& key, float& out) const {
    auto it = metadata.find(key);
    if (it == metadata.end()) return false;
    if (it->second.type == 6) {
        memcpy(&out, it->second.raw, 4);
        return true;
    }
    if (it->second.type == 12) {
        double d;
        memcpy(&d, it->second.raw, 8);
        out = float(d);
        return true;
    }
    int64_t i;
    if (get_int(key, i)) {
        out = float(i);
        return true;
    }
    return false;
}

bool GgufFile::get_string(const std::string& key, std::string& out) const {
    auto it = metadata.find(key);
    if (it == metadata.end() || it->second.type != 8) return false;
    uint64_t n;
    memcpy(&n, it->second.raw, 8);
    out.assign(reinterpret_cast<const char*>(it->second.raw + 8), n);
    return true;
}

bool GgufFile::get_int_array(const std::string& key, std::vector<int32_t>& out) const {
    auto it = metadata.find(key);
    if (it == metadata.end() || it->second.type != 9) return false;
    const GgufValue& v = it->second;
    if (v.elem != 4 && v.elem != 5) return false;
    out.resize(v.count);
    memcpy(out.data(), v.raw, v.count * 4);
    return true;
}

bool GgufFile::get_bool_array(const std::string& key, std::vector<bool>& out) const {
    auto it = metadata.find(key);
    if (it == metadata.end() || it->second.type != 9 || it->second.elem != 7) return false;
    out.resize(it->second.count);
    for (uint64_t i = 0; i < it->second.count; i++) out[i] = it->second.raw[i] != 0;
    return true;
}

bool GgufFile::get_float_array(const std::string& key, std::vector<float>& out) const {
    auto it = metadata.find(key);
    if (it == metadata.end() || it->second.type != 9 || it->second.elem != 6) return false;
    out.resize(it->second.count);
    memcpy(out.data(), it->second.raw, it->second.count * 4);
    return true;
}

bool GgufFile::get_bool(const std::string& key, bool& out) const {
    auto it = metadata.find(key);
    if (it == metadata.end() || it->second.type != 7) return false;
    out = it->second.raw[0] != 0;
    return true;
}

bool GgufFile::get_string_array(const std::string& key, std::vector<std::string>& out) const {
    auto it = metadata.find(key);
    if (it == metadata.end() || it->second.type != 9 || it->second.elem != 8) return false;
    // The directory walk in open() already checked every element against the file end.
    const uint8_t* p = it->second.raw;
    out.clear();
    out.reserve(it->second.count);
    for (uint64_t i = 0; i < it->second.count; i++) {
        uint64_t n;
        memcpy(&n, p, 8);
        out.emplace_back(reinterpret_cast<const char*>(p + 8), n);
        p += 8 + n;
    }
    return true;
}

bool GgufFile::get_string_array_count(const std::string& key, int64_t& out) const {
    auto it = metadata.find(key);
    if (it == metadata.end() || it->second.type != 9 || it->second.elem != 8) return false;
    out = int64_t(it->second.count);
    return true;
}

}  // namespace ge
