#include "tmap.h"

#include <mutex>

namespace m3r {

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    if (!fn) throw Error(kErrCuda, "cuTensorMapEncodeTiled is not available from the CUDA driver");
    return fn;
}

CUtensorMap encode(int dt, const void* ptr, int rank, const cuuint64_t* dims, const cuuint64_t* strides_bytes,
                   const cuuint32_t* box) {
    M3R_REQUIRE((reinterpret_cast<uintptr_t>(ptr) & 15) == 0, "tensor map base address must be 16-byte aligned");
    for (int i = 0; i < rank - 1; ++i)
        M3R_REQUIRE(strides_bytes[i] % 16 == 0, "tensor map strides must be multiples of 16 bytes");
    CUtensorMap m;
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    const CUtensorMapDataType type = dt == kTmapF32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                     : dt == 1      ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                    : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const CUresult r = encode_fn()(&m, type, rank, const_cast<void*>(ptr), dims, strides_bytes, box, estr,
                                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw Error(kErrCuda, "cuTensorMapEncodeTiled failed: " + std::to_string(int(r)));
    return m;
}

}  // namespace

CUtensorMap tmap_2d(int dt, const void* ptr, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows) {
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t str[1] = {ld * 2};
    const cuuint32_t box[2] = {64, box_rows};
    return encode(dt, ptr, 2, dims, str, box);
}

CUtensorMap tmap_2d_f32(const void* ptr, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows) {
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t str[1] = {ld * 4};
    const cuuint32_t box[2] = {32, box_rows};
    return encode(kTmapF32, ptr, 2, dims, str, box);
}

CUtensorMap tmap_3d_rows64(int dt, const void* ptr, uint64_t d1, uint64_t d2, uint32_t box_d1) {
    const cuuint64_t dims[3] = {64, d1, d2};
    const cuuint64_t str[2] = {64 * 2, d1 * 64 * 2};
    const cuuint32_t box[3] = {64, box_d1, 1};
    return encode(dt, ptr, 3, dims, str, box);
}

CUtensorMap tmap_nhwc(int dt, const void* ptr, uint64_t n, uint64_t h, uint64_t w, uint64_t c, uint64_t cstride,
                      uint32_t hbox, uint32_t wbox) {
    const cuuint64_t dims[4] = {c, w, h, n};
    const cuuint64_t str[3] = {cstride * 2, w * cstride * 2, h * w * cstride * 2};
    const cuuint32_t box[4] = {64, wbox, hbox, 1};
    return encode(dt, ptr, 4, dims, str, box);
}

}  // namespace m3r
