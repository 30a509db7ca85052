// Matcher arg-max for callers that cannot allocate device memory.
//
// Some callers of this library must not allocate GPU memory once they are running:
// a real-time loop (the drone / robot tracking use the reference targets) where the
// implicit device synchronisation of cudaMalloc / cudaFree would stall the frame
// pipeline, or a host framework that has already reserved all device memory in its
// own pool and forbids other allocators.  m3r_match_nn_static serves them: the
// caller passes device buffers for the inputs and the outputs, and every temporary
// buffer lives in one file-scope device array that the library reserves when it is
// loaded (every GPU that loads the library keeps it until the process exits).
//
// The array is shared by every call on a device and keeps the previous call's
// contents; the key buffers that must start at zero are cleared on the caller's
// stream by each call.  Calls that overlap on the GPU (same device, different
// streams, or a second call queued before the first has finished reading its
// outputs from the array) race on the array.
//
// The first call on a device looks up the array's device address with that device
// current (set-up); make that first call before any stream capture.
#include <mutex>
#include <string>

#include "../../include/m3r_cuda.h"
#include "matcher.h"
#include "tmap.h"

namespace {

// Limits of the shared scratch array: both descriptor sets up to 16384 rows, up to 64
// channels.  Layout: normalised A, normalised B (fp32), row keys, column keys (u64).
constexpr long long kMaxRows = 16384;
constexpr int kMaxDim = 64;
constexpr size_t kNormBytes = sizeof(float) * kMaxRows * kMaxDim;
constexpr size_t kKeyBytes = sizeof(unsigned long long) * kMaxRows;
constexpr size_t kScratchBytes = 2 * kNormBytes + 2 * kKeyBytes;  // 8.25 MiB

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_setup_mu;
void* g_scratch_addr[M3R_MAX_DEVICES] = {};

// Device address of g_noalloc_scratch on `device` (the current device), looked up once.
void* scratch_for(int device) {
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if (!g_scratch_addr[device]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p)
            throw m3r::Error(m3r::kErrCuda, std::string("cudaGetSymbolAddress(scratch) failed: ") + cudaGetErrorString(e));
        g_scratch_addr[device] = p;
    }
    return g_scratch_addr[device];
}

__global__ void decode_values_kernel(const unsigned long long* __restrict__ key, long long n, float* __restrict__ out) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const uint32_t k = static_cast<uint32_t>(key[i] >> 32);
        const uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
        out[i] = __uint_as_float(u);
    }
}

}  // namespace

namespace m3r {
void set_global_error(const std::string& msg);  // api.cpp: the text m3r_global_error() returns
}

extern "C" {

// Declared in include/m3r_cuda.h.
int m3r_match_nn_static(int device, const float* desc_1, const float* desc_2, int64_t n1, int64_t n2, int desc_dim,
                        int32_t* nn_12, int32_t* nn_21, float* best_12, void* stream) {
    try {
        if (!desc_1 || !desc_2 || !nn_12 || !nn_21 || n1 <= 0 || n2 <= 0 || desc_dim <= 0)
            throw m3r::Error(m3r::kErrArg, "match_nn_static: null buffer or non-positive size");
        if (n1 > kMaxRows || n2 > kMaxRows || desc_dim > kMaxDim)
            throw m3r::Error(m3r::kErrArg, "match_nn_static: sizes beyond the static scratch limit (rows <= " +
                                               std::to_string(kMaxRows) + " per set, desc_dim <= " +
                                               std::to_string(kMaxDim) + ")");
        if (device < 0 || device >= M3R_MAX_DEVICES) throw m3r::Error(m3r::kErrArg, "match_nn_static: bad device");
        int prev = 0;
        M3R_CUDA(cudaGetDevice(&prev));
        M3R_CUDA(cudaSetDevice(device));
        try {
            unsigned char* base = static_cast<unsigned char*>(scratch_for(device));
            float* a = reinterpret_cast<float*>(base);
            float* b = reinterpret_cast<float*>(base + kNormBytes);
            unsigned long long* rowkey = reinterpret_cast<unsigned long long*>(base + 2 * kNormBytes);
            unsigned long long* colkey = reinterpret_cast<unsigned long long*>(base + 2 * kNormBytes + kKeyBytes);
            cudaStream_t s = static_cast<cudaStream_t>(stream);
            m3r::match_normalize(s, desc_1, a, n1, desc_dim);
            m3r::match_normalize(s, desc_2, b, n2, desc_dim);
            // clears rowkey / colkey on the stream before merging into them
            m3r::match_argmax(s, a, b, 0, n1, n2, desc_dim, rowkey, colkey, true);
            m3r::match_decode(s, rowkey, n1, nn_12);
            m3r::match_decode(s, colkey, n2, nn_21);
            if (best_12) {
                const int blocks = static_cast<int>((n1 + 255) / 256 < 148 * 16 ? (n1 + 255) / 256 : 148 * 16);
                decode_values_kernel<<<blocks, 256, 0, s>>>(rowkey, n1, best_12);
                M3R_CUDA(cudaGetLastError());
            }
        } catch (...) {
            cudaSetDevice(prev);
            throw;
        }
        M3R_CUDA(cudaSetDevice(prev));
        return M3R_OK;
    } catch (const m3r::Error& x) {
        m3r::set_global_error(x.what());
        return x.code;
    } catch (const std::exception& x) {
        m3r::set_global_error(x.what());
        return M3R_ERR_CUDA;
    }
}

}  // extern "C"
