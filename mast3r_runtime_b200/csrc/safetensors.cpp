#include "safetensors.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>

#include "tmap.h"

namespace m3r {

namespace {

// A small recursive-descent JSON reader for the safetensors header:
// {"name": {"dtype": "F32", "shape": [..], "data_offsets": [b, e]}, "__metadata__": {...}}
struct Json {
    const char* p;
    const char* e;
    void ws() {
        while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
    }
    [[noreturn]] void fail(const char* what) { throw Error(kErrIo, std::string("safetensors header: ") + what); }
    void expect(char c) {
        ws();
        if (p >= e || *p != c) fail("unexpected character");
        ++p;
    }
    bool peek(char c) {
        ws();
        return p < e && *p == c;
    }
    std::string str() {
        expect('"');
        std::string s;
        while (p < e && *p != '"') {
            if (*p == '\\') {
                ++p;
                if (p >= e) fail("bad escape");
                if (*p == 'u') {  // keep escaped code units verbatim (names are ASCII in practice)
                    if (e - p < 5) fail("bad escape");
                    s.append(p - 1, 6);
                    p += 5;
                    continue;
                }
                s.push_back(*p == 'n' ? '\n' : *p == 't' ? '\t' : *p);
                ++p;
                continue;
            }
            s.push_back(*p++);
        }
        expect('"');
        return s;
    }
    int64_t integer() {
        ws();
        bool neg = false;
        if (p < e && *p == '-') {
            neg = true;
            ++p;
        }
        if (p >= e || *p < '0' || *p > '9') fail("expected integer");
        int64_t v = 0;
        while (p < e && *p >= '0' && *p <= '9') v = v * 10 + (*p++ - '0');
        return neg ? -v : v;
    }
    void skip_value() {
        ws();
        if (p >= e) fail("truncated");
        if (*p == '"') {
            str();
        } else if (*p == '{') {
            ++p;
            if (peek('}')) {
                ++p;
                return;
            }
            for (;;) {
                str();
                expect(':');
                skip_value();
                if (peek(',')) {
                    ++p;
                    continue;
                }
                expect('}');
                return;
            }
        } else if (*p == '[') {
            ++p;
            if (peek(']')) {
                ++p;
                return;
            }
            for (;;) {
                skip_value();
                if (peek(',')) {
                    ++p;
                    continue;
                }
                expect(']');
                return;
            }
        } else {
            while (p < e && *p != ',' && *p != '}' && *p != ']') ++p;
        }
    }
    std::vector<int64_t> int_list() {
        std::vector<int64_t> v;
        expect('[');
        if (peek(']')) {
            ++p;
            return v;
        }
        for (;;) {
            v.push_back(integer());
            if (peek(',')) {
                ++p;
                continue;
            }
            expect(']');
            return v;
        }
    }
};

float bf16_to_f32(uint16_t h) {
    uint32_t u = static_cast<uint32_t>(h) << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

float f16_to_f32(uint16_t h) {
    const uint32_t sign = (h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1F;
    uint32_t mant = h & 0x3FF;
    uint32_t u;
    if (exp == 0) {
        if (mant == 0) {
            u = sign;
        } else {  // subnormal
            exp = 127 - 15 + 1;
            while ((mant & 0x400) == 0) {
                mant <<= 1;
                --exp;
            }
            mant &= 0x3FF;
            u = sign | (exp << 23) | (mant << 13);
        }
    } else if (exp == 31) {
        u = sign | 0x7F800000u | (mant << 13);
    } else {
        u = sign | ((exp - 15 + 127) << 23) | (mant << 13);
    }
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

}  // namespace

SafetensorsFile::SafetensorsFile(const std::string& path) : path_(path) {
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) throw Error(kErrIo, "cannot open weights file: " + path);
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 8) {
        ::close(fd);
        throw Error(kErrIo, "weights file too small: " + path);
    }
    map_len_ = static_cast<size_t>(st.st_size);
    map_ = mmap(nullptr, map_len_, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (map_ == MAP_FAILED) {
        map_ = nullptr;
        throw Error(kErrIo, "mmap failed: " + path);
    }
    const uint8_t* base = static_cast<const uint8_t*>(map_);
    uint64_t hlen = 0;
    std::memcpy(&hlen, base, 8);
    if (hlen > map_len_ - 8) throw Error(kErrIo, "corrupt safetensors header length: " + path);
    data_ = base + 8 + hlen;
    data_len_ = map_len_ - 8 - hlen;
    Json j{reinterpret_cast<const char*>(base + 8), reinterpret_cast<const char*>(base + 8 + hlen)};
    j.expect('{');
    if (!j.peek('}')) {
        for (;;) {
            const std::string name = j.str();
            j.expect(':');
            if (name == "__metadata__") {
                j.skip_value();
            } else {
                TensorInfo ti;
                j.expect('{');
                for (;;) {
                    const std::string key = j.str();
                    j.expect(':');
                    if (key == "dtype") {
                        ti.dtype = j.str();
                    } else if (key == "shape") {
                        ti.shape = j.int_list();
                    } else if (key == "data_offsets") {
                        const auto o = j.int_list();
                        if (o.size() != 2 || o[0] < 0 || o[1] < o[0]) j.fail("bad data_offsets");
                        ti.begin = static_cast<uint64_t>(o[0]);
                        ti.end = static_cast<uint64_t>(o[1]);
                    } else {
                        j.skip_value();
                    }
                    if (j.peek(',')) {
                        ++j.p;
                        continue;
                    }
                    j.expect('}');
                    break;
                }
                if (ti.end > data_len_) throw Error(kErrIo, "tensor data out of file bounds: " + name);
                tensors_[name] = ti;
            }
            if (j.peek(',')) {
                ++j.p;
                continue;
            }
            j.expect('}');
            break;
        }
    } else {
        ++j.p;
    }
}

SafetensorsFile::~SafetensorsFile() {
    if (map_) munmap(map_, map_len_);
}

const TensorInfo& SafetensorsFile::info(const std::string& name) const {
    auto it = tensors_.find(name);
    if (it == tensors_.end()) throw Error(kErrIo, "missing tensor in " + path_ + ": " + name);
    return it->second;
}

std::vector<float> SafetensorsFile::load_f32(const std::string& name, const std::vector<int64_t>& expect) const {
    const TensorInfo& ti = info(name);
    if (!expect.empty() && ti.shape != expect) {
        std::string got, want;
        for (auto d : ti.shape) got += std::to_string(d) + ",";
        for (auto d : expect) want += std::to_string(d) + ",";
        throw Error(kErrIo, "tensor " + name + " has shape [" + got + "], expected [" + want + "]");
    }
    const int64_t n = ti.numel();
    std::vector<float> out(static_cast<size_t>(n));
    const uint8_t* src = data_ + ti.begin;
    const uint64_t bytes = ti.end - ti.begin;
    if (ti.dtype == "F32") {
        if (bytes != static_cast<uint64_t>(n) * 4) throw Error(kErrIo, "size mismatch for " + name);
        std::memcpy(out.data(), src, bytes);
    } else if (ti.dtype == "BF16" || ti.dtype == "F16") {
        if (bytes != static_cast<uint64_t>(n) * 2) throw Error(kErrIo, "size mismatch for " + name);
        const bool bf = ti.dtype == "BF16";
        for (int64_t i = 0; i < n; ++i) {
            uint16_t h;
            std::memcpy(&h, src + 2 * i, 2);
            out[static_cast<size_t>(i)] = bf ? bf16_to_f32(h) : f16_to_f32(h);
        }
    } else {
        throw Error(kErrIo, "unsupported dtype " + ti.dtype + " for " + name);
    }
    return out;
}

}  // namespace m3r
