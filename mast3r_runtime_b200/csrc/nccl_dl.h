// NCCL, loaded at run time (dlopen "libnccl.so.2"), so that the library loads and its
// single-device paths work on hosts without NCCL.  Only the calls the multi-device
// matcher needs are resolved.
#pragma once

#include <nccl.h>

#include <string>

namespace m3r {

struct NcclApi {
    ncclResult_t (*CommInitAll)(ncclComm_t*, int, const int*) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

// The resolved API; throws Error(kErrNccl) when NCCL cannot be loaded.
const NcclApi& nccl();

// Throws Error(kErrNccl) with the call's text when r is not ncclSuccess.
void nccl_check(ncclResult_t r, const char* what);

}  // namespace m3r
