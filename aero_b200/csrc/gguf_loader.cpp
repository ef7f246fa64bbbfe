// GGUF reader for the device loader: mmap the file, parse the header, the
// metadata and the tensor index, and hand out pointers into the mapping.
//
// Container layout as the reference reads it (engine/gguf.py:1-19,
// src/gguf.cpp:150-275): magic "GGUF", u32 version (2 or 3), u64 tensor count,
// u64 kv count, kv pairs, tensor infos (name, u32 n_dims, u64 dims fastest
// first, u32 type, u64 offset from the data section), padding to
// general.alignment (default 32, a power of two), data. Every read is bounds
// checked against the file size, so a truncated file is refused, not overread.
#include "gguf_loader.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>

namespace aero {

namespace {
enum : uint32_t {
    V_U8 = 0, V_I8, V_U16, V_I16, V_U32, V_I32, V_F32, V_BOOL, V_STR, V_ARR, V_U64, V_I64, V_F64
};
size_t scalar_size(uint32_t t) {
    switch (t) {
        case V_U8: case V_I8: case V_BOOL: return 1;
        case V_U16: case V_I16: return 2;
        case V_U32: case V_I32: case V_F32: return 4;
        case V_U64: case V_I64: case V_F64: return 8;
    }
    return 0;
}
}  // namespace

struct Cursor {
    const uint8_t* p;
    size_t n, off = 0;
    bool ok = true;
    bool need(size_t k) {
        if (!ok || off + k > n) ok = false;
        return ok;
    }
    uint32_t u32() {
        if (!need(4)) return 0;
        uint32_t v;
        std::memcpy(&v, p + off, 4);
        off += 4;
        return v;
    }
    uint64_t u64() {
        if (!need(8)) return 0;
        uint64_t v;
        std::memcpy(&v, p + off, 8);
        off += 8;
        return v;
    }
    std::string str() {
        const uint64_t len = u64();
        if (len > (1u << 30) || !need(len)) {
            ok = false;
            return {};
        }
        std::string s(reinterpret_cast<const char*>(p + off), len);
        off += len;
        return s;
    }
    // Reads one value of type t; integers are also returned in *iv when set.
    bool value(uint32_t t, int64_t* iv, std::string* sv, int depth = 0) {
        if (depth > 4) return ok = false;
        if (t == V_STR) {
            std::string s = str();
            if (sv) *sv = s;
            return ok;
        }
        if (t == V_ARR) {
            const uint32_t et = u32();
            const uint64_t cnt = u64();
            if (!ok) return false;
            const size_t es = scalar_size(et);
            if (es) {
                if (cnt > n || !need(cnt * es)) return ok = false;
                off += cnt * es;
                return true;
            }
            for (uint64_t i = 0; i < cnt && ok; ++i) value(et, nullptr, nullptr, depth + 1);
            return ok;
        }
        const size_t sz = scalar_size(t);
        if (!sz || !need(sz)) return ok = false;
        int64_t v = 0;
        switch (t) {
            case V_U8: v = p[off]; break;
            case V_I8: v = (int8_t)p[off]; break;
            case V_U16: { uint16_t x; std::memcpy(&x, p + off, 2); v = x; break; }
            case V_I16: { int16_t x; std::memcpy(&x, p + off, 2); v = x; break; }
            case V_U32: { uint32_t x; std::memcpy(&x, p + off, 4); v = x; break; }
            case V_I32: { int32_t x; std::memcpy(&x, p + off, 4); v = x; break; }
            case V_U64: { uint64_t x; std::memcpy(&x, p + off, 8); v = (int64_t)x; break; }
            case V_I64: { int64_t x; std::memcpy(&x, p + off, 8); v = x; break; }
            case V_BOOL: v = p[off] ? 1 : 0; break;
            default: v = 0;
        }
        off += sz;
        if (iv) *iv = v;
        return true;
    }
};

GgufFile::~GgufFile() {
    if (map_ && map_ != MAP_FAILED) munmap(const_cast<uint8_t*>(map_), size_);
}

bool GgufFile::open(const std::string& path, std::string* err) {
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) {
        *err = path + ": cannot open";
        return false;
    }
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 24) {
        ::close(fd);
        *err = path + ": not a GGUF file (too short)";
        return false;
    }
    size_ = (size_t)st.st_size;
    void* m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (m == MAP_FAILED) {
        *err = path + ": mmap failed";
        return false;
    }
    map_ = static_cast<const uint8_t*>(m);
    Cursor c{map_, size_};
    if (std::memcmp(map_, "GGUF", 4) != 0) {
        *err = path + ": not a GGUF file (bad magic)";
        return false;
    }
    c.off = 4;
    version_ = c.u32();
    if (version_ != 2 && version_ != 3) {
        *err = path + ": unsupported GGUF version " + std::to_string(version_);
        return false;
    }
    const uint64_t n_tensors = c.u64(), n_kv = c.u64();
    if (n_tensors > (1u << 24) || n_kv > (1u << 24)) {
        *err = path + ": implausible tensor/kv counts";
        return false;
    }
    for (uint64_t i = 0; i < n_kv && c.ok; ++i) {
        const std::string key = c.str();
        const uint32_t t = c.u32();
        int64_t iv = 0;
        std::string sv;
        const bool has_int = t != V_STR && t != V_ARR && t != V_F32 && t != V_F64;
        const size_t at = c.off;
        c.value(t, &iv, &sv);
        if (has_int) ints_[key] = iv;
        if (t == V_STR) strs_[key] = sv;
        if (c.ok && t == V_F32) {
            float f;
            std::memcpy(&f, map_ + at, 4);
            floats_[key] = f;
        } else if (c.ok && t == V_F64) {
            double f;
            std::memcpy(&f, map_ + at, 8);
            floats_[key] = f;
        }
    }
    if (!c.ok) {
        *err = path + ": truncated metadata";
        return false;
    }
    alignment_ = 32;
    auto it = ints_.find("general.alignment");
    if (it != ints_.end()) alignment_ = (uint64_t)it->second;
    if (alignment_ == 0 || (alignment_ & (alignment_ - 1))) {
        *err = path + ": bad alignment (must be a power of two)";
        return false;
    }
    for (uint64_t i = 0; i < n_tensors && c.ok; ++i) {
        GgufTensor ti;
        ti.name = c.str();
        const uint32_t nd = c.u32();
        if (nd == 0 || nd > 4) {
            c.ok = false;
            break;
        }
        ti.n_values = 1;
        for (uint32_t k = 0; k < nd; ++k) {
            const uint64_t dim = c.u64();
            ti.dims.push_back((int64_t)dim);
            ti.n_values *= (int64_t)dim;
        }
        ti.type = (int)c.u32();
        ti.offset = c.u64();
        tensors_[ti.name] = ti;
    }
    if (!c.ok) {
        *err = path + ": truncated tensor index";
        return false;
    }
    data_off_ = (c.off + alignment_ - 1) / alignment_ * alignment_;
    for (auto& kv : tensors_) {
        GgufTensor& t = kv.second;
        const int64_t bb = t.type == 8 ? 34 : t.type == 12 ? 144 : t.type == 0 ? 4 : t.type == 1 ? 2 : 0;
        const int64_t bv = t.type == 8 ? 32 : t.type == 12 ? 256 : 1;
        t.nbytes = bb > 0 && t.n_values % bv == 0 ? t.n_values / bv * bb : -1;
        if (t.nbytes >= 0 && (data_off_ + t.offset + (uint64_t)t.nbytes > size_)) {
            *err = path + ": tensor " + t.name + " extends past the end of the file";
            return false;
        }
    }
    return true;
}

const GgufTensor* GgufFile::find(const std::string& name) const {
    auto it = tensors_.find(name);
    return it == tensors_.end() ? nullptr : &it->second;
}

const uint8_t* GgufFile::data(const GgufTensor& t) const { return map_ + data_off_ + t.offset; }

bool GgufFile::get_int(const std::string& key, int64_t* v) const {
    auto it = ints_.find(key);
    if (it == ints_.end()) return false;
    *v = it->second;
    return true;
}

bool GgufFile::get_float(const std::string& key, double* v) const {
    auto it = floats_.find(key);
    if (it == floats_.end()) return false;
    *v = it->second;
    return true;
}

std::string GgufFile::arch() const {
    auto it = strs_.find("general.architecture");
    return it == strs_.end() ? std::string("unknown") : it->second;
}

}  // namespace aero
