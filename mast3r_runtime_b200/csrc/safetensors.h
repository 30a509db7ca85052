// Minimal safetensors reader (F32 / F16 / BF16), the checkpoint format the
// reference loads (csrc/common/safetensors.hpp:264-410 of the reference).
#pragma once

#include <stdint.h>

#include <map>
#include <string>
#include <vector>

namespace m3r {

struct TensorInfo {
    std::string dtype;
    std::vector<int64_t> shape;
    uint64_t begin = 0, end = 0;  // byte offsets into the data section
    int64_t numel() const {
        int64_t n = 1;
        for (int64_t d : shape) n *= d;
        return n;
    }
};

class SafetensorsFile {
public:
    explicit SafetensorsFile(const std::string& path);
    ~SafetensorsFile();
    SafetensorsFile(const SafetensorsFile&) = delete;
    SafetensorsFile& operator=(const SafetensorsFile&) = delete;

    bool has(const std::string& name) const { return tensors_.count(name) != 0; }
    const TensorInfo& info(const std::string& name) const;
    // Tensor as float32 (converted from F16 / BF16); throws when the shape differs from `expect`
    // (an empty `expect` accepts any shape).
    std::vector<float> load_f32(const std::string& name, const std::vector<int64_t>& expect = {}) const;
    const std::map<std::string, TensorInfo>& tensors() const { return tensors_; }

private:
    std::map<std::string, TensorInfo> tensors_;
    const uint8_t* data_ = nullptr;  // start of the data section (mmap)
    void* map_ = nullptr;
    size_t map_len_ = 0;
    uint64_t data_len_ = 0;
    std::string path_;
};

}  // namespace m3r
