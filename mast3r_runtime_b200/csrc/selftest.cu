// Self-test of the bounded device waits that every tcgen05 kernel of the library uses
// (mbar_wait, common.cuh): one warp waits on an mbarrier that nothing ever signals,
// with a caller-chosen limit.  The wait gives up after the limit, records its code in
// the device status block and the kernel returns, so the failure path of a stuck
// pipeline (a TMA load or an MMA that never completes) is exercised without faulting
// or hanging the GPU: the context stays usable for the next launch.
#include <string>

#include "../../include/m3r_cuda.h"
#include "common.cuh"
#include "engine.h"
#include "tmap.h"

namespace m3r {
void set_global_error(const std::string& msg);  // api.cpp: the text m3r_global_error() returns
}

namespace {

__global__ void never_signalled_wait_kernel(int* status) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        m3r::mbar_init(&bar, 1);  // one arrival expected; none comes
        abort_flag = 0;
        m3r::fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) m3r::mbar_wait(&bar, 0, &abort_flag, m3r::kDevTimeoutMma, status);
    __syncthreads();
}

}  // namespace

extern "C" {

// Declared in include/m3r_cuda.h.
int m3r_wait_selftest(int device, unsigned long long limit_ns, int* device_code) {
    try {
        if (device_code) *device_code = 0;
        if (limit_ns == 0 || limit_ns > 10000000000ull)
            throw m3r::Error(m3r::kErrArg, "wait_selftest: limit must be in (0, 10 s]");
        m3r::DeviceGuard g(device);
        m3r::DevStatus* st = nullptr;
        M3R_CUDA(cudaMalloc(&st, sizeof(m3r::DevStatus)));
        m3r::DevStatus init{0, 0, limit_ns};
        int code = 0;
        try {
            M3R_CUDA(cudaMemcpy(st, &init, sizeof(init), cudaMemcpyHostToDevice));
            never_signalled_wait_kernel<<<1, 32>>>(reinterpret_cast<int*>(st));
            M3R_CUDA(cudaGetLastError());
            M3R_CUDA(cudaDeviceSynchronize());
            M3R_CUDA(cudaMemcpy(&code, st, sizeof(int), cudaMemcpyDeviceToHost));
        } catch (...) {
            cudaFree(st);
            throw;
        }
        cudaFree(st);
        if (device_code) *device_code = code;
        if (code != 0)
            throw m3r::Error(m3r::kErrTimeout, "device wait timed out (code " + std::to_string(code) + ")");
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
