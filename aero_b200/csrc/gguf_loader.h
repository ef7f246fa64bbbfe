// mmap GGUF reader used by aero_cuda_moe_open_gguf.
#pragma once
#include <stddef.h>
#include <stdint.h>

#include <map>
#include <string>
#include <vector>

namespace aero {

struct GgufTensor {
    std::string name;
    std::vector<int64_t> dims;  // GGUF order, fastest-varying first
    int type = -1;              // ggml type id
    uint64_t offset = 0;        // from the data section
    int64_t n_values = 0;
    int64_t nbytes = -1;        // -1 for a type this library does not read
    // row-major shape: dims reversed
    int64_t shape(int i) const { return dims[dims.size() - 1 - (size_t)i]; }
};

class GgufFile {
public:
    GgufFile() = default;
    ~GgufFile();
    GgufFile(const GgufFile&) = delete;
    GgufFile& operator=(const GgufFile&) = delete;

    bool open(const std::string& path, std::string* err);
    const GgufTensor* find(const std::string& name) const;
    const uint8_t* data(const GgufTensor& t) const;
    bool get_int(const std::string& key, int64_t* v) const;
    bool get_float(const std::string& key, double* v) const;  // F32 / F64 values
    std::string arch() const;
    uint64_t alignment() const { return alignment_; }

private:
    const uint8_t* map_ = nullptr;
    size_t size_ = 0;
    uint32_t version_ = 0;
    uint64_t alignment_ = 32, data_off_ = 0;
    std::map<std::string, int64_t> ints_;
    std::map<std::string, double> floats_;
    std::map<std::string, std::string> strs_;
    std::map<std::string, GgufTensor> tensors_;
};

}  // namespace aero
