// Host-side TMA tensor-map encoding (cuTensorMapEncodeTiled through the runtime's
// driver entry point, so the library does not link libcuda directly).  All maps
// use 128-byte swizzled boxes whose inner extent is 128 bytes (64 16-bit or 32
// fp32 elements); out-of-bounds box elements read as zero and are not stored.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>

namespace m3r {

struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

// Status codes of the C ABI (include/m3r_cuda.h)
constexpr int kOk = 0;
constexpr int kErrArg = -1;
constexpr int kErrIo = -2;
constexpr int kErrCuda = -3;
constexpr int kErrNccl = -4;
constexpr int kErrTimeout = -5;
constexpr int kErrState = -6;
constexpr int kErrNoMem = -7;

#define M3R_CUDA(call)                                                                                 \
    do {                                                                                               \
        cudaError_t e_ = (call);                                                                       \
        if (e_ != cudaSuccess)                                                                         \
            throw ::m3r::Error(e_ == cudaErrorMemoryAllocation ? ::m3r::kErrNoMem : ::m3r::kErrCuda,   \
                               std::string(#call) + ": " + cudaGetErrorString(e_) + " (" + __FILE__ + \
                                   ":" + std::to_string(__LINE__) + ")");                              \
    } while (0)

#define M3R_REQUIRE(cond, msg)                                            \
    do {                                                                  \
        if (!(cond)) throw ::m3r::Error(::m3r::kErrArg, std::string(msg)); \
    } while (0)

// Element type code of the fp32 maps (the 16-bit maps take a Dt code: 0 bf16, 1 fp16).
constexpr int kTmapF32 = 2;

// row-major matrix [rows, cols] with row stride ld (elements); box [box_rows, 64].
CUtensorMap tmap_2d(int dt, const void* ptr, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows);

// row-major fp32 matrix [rows, cols], row stride ld (elements); box [box_rows, 32].
CUtensorMap tmap_2d_f32(const void* ptr, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows);

// tensor [d2, d1, 64] (innermost 64 = head dim), box [box_d1, 64].
CUtensorMap tmap_3d_rows64(int dt, const void* ptr, uint64_t d1, uint64_t d2, uint32_t box_d1);

// NHWC tensor [n, h, w, c] (pixel stride cstride elements), box [1, hbox, wbox, 64].
CUtensorMap tmap_nhwc(int dt, const void* ptr, uint64_t n, uint64_t h, uint64_t w, uint64_t c, uint64_t cstride,
                      uint32_t hbox, uint32_t wbox);

}  // namespace m3r
