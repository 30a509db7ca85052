// C ABI (include/m3r_cuda.h): argument checks, exception -> status code mapping,
// per-engine and thread-local last-error strings.
#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/m3r_cuda.h"
#include "attention.h"
#include "common.cuh"
#include "engine.h"
#include "gemm.h"
#include "kernels.h"
#include "matcher.h"

struct m3r_engine {
    m3r::Engine* impl = nullptr;
    std::string err;
};

namespace {

thread_local std::string g_err;

template <class F>
int guarded(m3r_engine* e, F&& fn) {
    try {
        fn();
        (e ? e->err : g_err).clear();
        return M3R_OK;
    } catch (const m3r::Error& x) {
        (e ? e->err : g_err) = x.what();
        return x.code;
    } catch (const std::bad_alloc&) {
        (e ? e->err : g_err) = "host allocation failed";
        return M3R_ERR_NOMEM;
    } catch (const std::exception& x) {
        (e ? e->err : g_err) = x.what();
        return M3R_ERR_CUDA;
    }
}

// Device buffer owned for the duration of one test-entry call.
struct DBuf {
    void* p = nullptr;
    explicit DBuf(size_t bytes) { M3R_CUDA(cudaMalloc(&p, bytes > 0 ? bytes : 16)); }
    ~DBuf() {
        if (p) cudaFree(p);
    }
    template <class T>
    T* as() const {
        return static_cast<T*>(p);
    }
};

struct Events {
    cudaEvent_t a, b;
    Events() {
        M3R_CUDA(cudaEventCreate(&a));
        M3R_CUDA(cudaEventCreate(&b));
    }
    ~Events() {
        cudaEventDestroy(a);
        cudaEventDestroy(b);
    }
    float ms() const {
        float t = 0;
        M3R_CUDA(cudaEventElapsedTime(&t, a, b));
        return t;
    }
};

void check_dev_err(int* d_err) {
    int e = 0;
    M3R_CUDA(cudaMemcpy(&e, d_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (e) throw m3r::Error(m3r::kErrTimeout, "device wait timed out (code " + std::to_string(e) + ")");
}

}  // namespace

namespace m3r {
// Lets entry points defined outside this file report through m3r_global_error().
void set_global_error(const std::string& msg) { g_err = msg; }
}  // namespace m3r

extern "C" {

int m3r_version(void) { return M3R_ABI_VERSION; }

const char* m3r_global_error(void) { return g_err.c_str(); }

int m3r_device_count(int* count) {
    return guarded(nullptr, [&] {
        M3R_REQUIRE(count != nullptr, "count is null");
        int n = 0;
        const cudaError_t e = cudaGetDeviceCount(&n);
        if (e != cudaSuccess) {
            cudaGetLastError();
            n = 0;
        }
        *count = n;
    });
}

int m3r_device_info(int device, char* name, int name_len, int* cc_major, int* cc_minor) {
    return guarded(nullptr, [&] {
        cudaDeviceProp prop;
        M3R_CUDA(cudaGetDeviceProperties(&prop, device));
        if (name && name_len > 0) {
            std::strncpy(name, prop.name, static_cast<size_t>(name_len) - 1);
            name[name_len - 1] = '\0';
        }
        if (cc_major) *cc_major = prop.major;
        if (cc_minor) *cc_minor = prop.minor;
    });
}

int m3r_create(const m3r_config* cfg, m3r_engine** out) {
    return guarded(nullptr, [&] {
        M3R_REQUIRE(cfg != nullptr && out != nullptr, "null argument");
        *out = nullptr;
        auto* e = new m3r_engine();
        try {
            e->impl = new m3r::Engine(*cfg);
        } catch (...) {
            delete e;
            throw;
        }
        *out = e;
    });
}

void m3r_destroy(m3r_engine* engine) {
    if (!engine) return;
    try {
        delete engine->impl;
    } catch (...) {
    }
    delete engine;
}

const char* m3r_last_error(const m3r_engine* engine) { return engine ? engine->err.c_str() : g_err.c_str(); }

int m3r_load(m3r_engine* engine, const char* path) {
    if (!engine) return M3R_ERR_ARG;
    return guarded(engine, [&] {
        M3R_REQUIRE(path != nullptr, "path is null");
        engine->impl->load(path);
    });
}

int m3r_check_checkpoint(const m3r_config* cfg, const char* path) {
    return guarded(nullptr, [&] {
        M3R_REQUIRE(cfg != nullptr && path != nullptr, "null argument");
        m3r::check_checkpoint(path, m3r::Dims::from(*cfg));
    });
}

int m3r_is_ready(const m3r_engine* engine) { return engine && engine->impl && engine->impl->ready() ? 1 : 0; }

int m3r_infer(m3r_engine* engine, const uint8_t* img1, const uint8_t* img2, int n_pairs, float* pts3d_1,
              float* pts3d_2, float* desc_1, float* desc_2, float* conf_1, float* conf_2, float* timing_ms) {
    if (!engine) return M3R_ERR_ARG;
    return guarded(engine, [&] {
        M3R_REQUIRE(img1 && img2 && n_pairs >= 1, "infer: null image or n_pairs < 1");
        float* outs[6] = {pts3d_1, pts3d_2, desc_1, desc_2, conf_1, conf_2};
        engine->impl->infer(img1, img2, n_pairs, outs, timing_ms);
    });
}

int m3r_infer_any(m3r_engine* engine, const uint8_t* img1, int h1, int w1, const uint8_t* img2, int h2, int w2,
                  float* pts3d_1, float* pts3d_2, float* desc_1, float* desc_2, float* conf_1, float* conf_2,
                  float* timing_ms) {
    if (!engine) return M3R_ERR_ARG;
    return guarded(engine, [&] {
        float* outs[6] = {pts3d_1, pts3d_2, desc_1, desc_2, conf_1, conf_2};
        engine->impl->infer_any(img1, h1, w1, img2, h2, w2, outs, timing_ms);
    });
}

int m3r_load_retrieval(m3r_engine* engine, const char* path) {
    if (!engine) return M3R_ERR_ARG;
    return guarded(engine, [&] {
        M3R_REQUIRE(path != nullptr, "path is null");
        engine->impl->load_retrieval(path);
    });
}

int m3r_encode_retrieval(m3r_engine* engine, const uint8_t* images, int n_images, float* features, float* attention,
                         float* timing_ms) {
    if (!engine) return M3R_ERR_ARG;
    return guarded(engine, [&] { engine->impl->encode_retrieval(images, n_images, features, attention, timing_ms); });
}

int m3r_resize_crop_test(int device, const uint8_t* src, int h, int w, uint8_t* dst, int out_h, int out_w) {
    return guarded(nullptr, [&] {
        M3R_REQUIRE(src && dst && h > 0 && w > 0 && out_h > 0 && out_w > 0, "resize_crop_test: bad arguments");
        m3r::DeviceGuard g(device);
        const size_t bi = static_cast<size_t>(h) * w * 3, bo = static_cast<size_t>(out_h) * out_w * 3;
        DBuf din(bi), dout(bo);
        M3R_CUDA(cudaMemcpy(din.p, src, bi, cudaMemcpyHostToDevice));
        m3r::resize_crop(nullptr, din.as<uint8_t>(), h, w, dout.as<uint8_t>(), out_h, out_w);
        M3R_CUDA(cudaDeviceSynchronize());
        M3R_CUDA(cudaMemcpy(dst, dout.p, bo, cudaMemcpyDeviceToHost));
    });
}

int m3r_resize2x_test(int device, int dtype, const uint16_t* x, int n, int h, int w, int c, uint16_t* y) {
    return guarded(nullptr, [&] {
        M3R_REQUIRE(x && y && n > 0 && h > 0 && w > 0 && c > 0 && c % 8 == 0, "resize2x_test: bad arguments");
        m3r::DeviceGuard g(device);
        const size_t bi = static_cast<size_t>(n) * h * w * c * 2, bo = 4 * bi;
        DBuf din(bi), dout(bo);
        M3R_CUDA(cudaMemcpy(din.p, x, bi, cudaMemcpyHostToDevice));
        m3r::resize16(nullptr, dtype, din.p, n, h, w, c, 2 * h, 2 * w, dout.p);
        M3R_CUDA(cudaDeviceSynchronize());
        M3R_CUDA(cudaMemcpy(y, dout.p, bo, cudaMemcpyDeviceToHost));
    });
}

int m3r_dpt_fuse_test(int device, int dtype, const uint16_t* f0, const uint16_t* f1, int h1, int w1,
                      const uint16_t* f2, int h2, int w2, const uint16_t* f3, int h3, int w3, int n, int H, int W,
                      int c, uint16_t* out) {
    return guarded(nullptr, [&] {
        M3R_REQUIRE(f0 && f1 && f2 && f3 && out && n > 0 && H > 0 && W > 0 && h1 > 0 && w1 > 0 && h2 > 0 &&
                        w2 > 0 && h3 > 0 && w3 > 0 && c > 0 && c % 8 == 0,
                    "dpt_fuse_test: bad arguments");
        m3r::DeviceGuard g(device);
        const size_t e = static_cast<size_t>(n) * c * 2;
        const size_t b0 = e * H * W, b1 = e * h1 * w1, b2 = e * h2 * w2, b3 = e * h3 * w3;
        DBuf d0(b0), d1(b1), d2(b2), d3(b3), dout(b0);
        M3R_CUDA(cudaMemcpy(d0.p, f0, b0, cudaMemcpyHostToDevice));
        M3R_CUDA(cudaMemcpy(d1.p, f1, b1, cudaMemcpyHostToDevice));
        M3R_CUDA(cudaMemcpy(d2.p, f2, b2, cudaMemcpyHostToDevice));
        M3R_CUDA(cudaMemcpy(d3.p, f3, b3, cudaMemcpyHostToDevice));
        m3r::dpt_fuse(nullptr, dtype, d0.p, d1.p, h1, w1, d2.p, h2, w2, d3.p, h3, w3, n, H, W, c, dout.p);
        M3R_CUDA(cudaDeviceSynchronize());
        M3R_CUDA(cudaMemcpy(out, dout.p, b0, cudaMemcpyDeviceToHost));
    });
}

int m3r_match(m3r_engine* engine, const float* desc_1, const float* desc_2, int height, int width, int desc_dim,
              int top_k, int reciprocal, float confidence_threshold, int64_t* idx_1, int64_t* idx_2,
              float* confidence, float* pts2d_1, float* pts2d_2, int* n_matches, float* timing_ms) {
    if (!engine) return M3R_ERR_ARG;
    return guarded(engine, [&] {
        M3R_REQUIRE(n_matches != nullptr, "n_matches is null");
        *n_matches = 0;
        const long long n = static_cast<long long>(height) * width;
        M3R_REQUIRE(n == 0 || (desc_1 && desc_2 && idx_1 && idx_2 && confidence && pts2d_1 && pts2d_2),
                    "match: null buffer");
        *n_matches = engine->impl->match(desc_1, desc_2, height, width, desc_dim, top_k, reciprocal,
                                         confidence_threshold, idx_1, idx_2, confidence, pts2d_1, pts2d_2, timing_ms);
    });
}

int m3r_match_ex(m3r_engine* engine, const float* desc_1, const float* desc_2, const float* conf_1,
                 const float* conf_2, const float* pts3d_1, const float* pts3d_2, int height, int width, int desc_dim,
                 int top_k, int reciprocal, float confidence_threshold, int64_t* idx_1, int64_t* idx_2,
                 float* confidence, float* pts2d_1, float* pts2d_2, float* match_pts3d_1, float* match_pts3d_2,
                 int* n_matches, float* timing_ms) {
    if (!engine) return M3R_ERR_ARG;
    return guarded(engine, [&] {
        M3R_REQUIRE(n_matches != nullptr, "n_matches is null");
        *n_matches = 0;
        const long long n = static_cast<long long>(height) * width;
        M3R_REQUIRE(n == 0 || (desc_1 && desc_2 && idx_1 && idx_2 && confidence && pts2d_1 && pts2d_2),
                    "match: null buffer");
        M3R_REQUIRE((conf_1 == nullptr) == (conf_2 == nullptr), "match: give both confidence maps or neither");
        M3R_REQUIRE((match_pts3d_1 == nullptr) == (match_pts3d_2 == nullptr), "match: give both pts3d outputs or neither");
        m3r::MatchExtras ex;
        ex.conf_1 = conf_1;
        ex.conf_2 = conf_2;
        ex.pts3d_1 = pts3d_1;
        ex.pts3d_2 = pts3d_2;
        ex.out3_1 = match_pts3d_1;
        ex.out3_2 = match_pts3d_2;
        *n_matches = engine->impl->match(desc_1, desc_2, height, width, desc_dim, top_k, reciprocal,
                                         confidence_threshold, idx_1, idx_2, confidence, pts2d_1, pts2d_2, timing_ms,
                                         &ex);
    });
}

int m3r_stage_inputs(m3r_engine* engine, const uint8_t* img1, const uint8_t* img2, int n_pairs) {
    if (!engine) return M3R_ERR_ARG;
    return guarded(engine, [&] {
        M3R_REQUIRE(img1 && img2, "null image");
        engine->impl->stage(img1, img2, n_pairs);
    });
}

int m3r_run_resident(m3r_engine* engine, int n_pairs, float* device_ms) {
    if (!engine) return M3R_ERR_ARG;
    return guarded(engine, [&] {
        const float ms = engine->impl->run_resident(n_pairs, nullptr);
        if (device_ms) *device_ms = ms;
    });
}

int m3r_fetch_outputs(m3r_engine* engine, int n_pairs, float* pts3d_1, float* pts3d_2, float* desc_1,
                      float* desc_2, float* conf_1, float* conf_2) {
    if (!engine) return M3R_ERR_ARG;
    return guarded(engine, [&] {
        float* outs[6] = {pts3d_1, pts3d_2, desc_1, desc_2, conf_1, conf_2};
        engine->impl->fetch(n_pairs, outs);
    });
}

int m3r_set_profiling(m3r_engine* engine, int on) {
    if (!engine) return M3R_ERR_ARG;
    engine->impl->set_profiling(on != 0);
    return M3R_OK;
}

int m3r_set_wait_timeout(m3r_engine* engine, unsigned long long ns) {
    if (!engine) return M3R_ERR_ARG;
    return guarded(engine, [&] { engine->impl->set_wait_timeout(ns); });
}

int m3r_get_profile(const m3r_engine* engine, double* out8) {
    if (!engine || !out8) return M3R_ERR_ARG;
    engine->impl->profile(out8);
    return M3R_OK;
}

int m3r_get_profile_ops(const m3r_engine* engine, char* buf, int cap, int* needed) {
    if (!engine || (cap > 0 && !buf)) return M3R_ERR_ARG;
    const std::string t = engine->impl->profile_ops();
    if (needed) *needed = static_cast<int>(t.size()) + 1;
    if (cap > 0) {
        const size_t n = std::min(t.size(), static_cast<size_t>(cap - 1));
        std::memcpy(buf, t.data(), n);
        buf[n] = '\0';
    }
    return M3R_OK;
}

void* m3r_host_alloc(size_t bytes) {
    void* p = nullptr;
    if (cudaHostAlloc(&p, bytes > 0 ? bytes : 16, cudaHostAllocPortable) != cudaSuccess) {
        cudaGetLastError();
        g_err = "cudaHostAlloc failed";
        return nullptr;
    }
    return p;
}

void m3r_host_free(void* p) {
    if (p) cudaFreeHost(p);
}

int m3r_attention_fwd(int device, int dtype, const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out,
                      int n_seq, int heads, int nq, int nk, float scale, int iters, float* kernel_ms) {
    return guarded(nullptr, [&] {
        M3R_REQUIRE(q && k && v && out && n_seq > 0 && heads > 0 && nq > 0 && nk > 0, "attention: bad arguments");
        m3r::DeviceGuard g(device);
        const size_t qn = static_cast<size_t>(n_seq) * heads * nq * 64, kn = static_cast<size_t>(n_seq) * heads * nk * 64;
        DBuf dq(qn * 2), dk(kn * 2), dv(kn * 2), dout(qn * 2), derr(sizeof(m3r::DevStatus));
        M3R_CUDA(cudaMemcpy(dq.p, q, qn * 2, cudaMemcpyHostToDevice));
        M3R_CUDA(cudaMemcpy(dk.p, k, kn * 2, cudaMemcpyHostToDevice));
        M3R_CUDA(cudaMemcpy(dv.p, v, kn * 2, cudaMemcpyHostToDevice));
        M3R_CUDA(cudaMemset(derr.p, 0, sizeof(m3r::DevStatus)));
        const int it = iters < 1 ? 1 : iters;
        Events ev;
        m3r::attention_fwd(nullptr, dtype, dq.p, dk.p, dv.p, dout.p, n_seq, heads, nq, nk, scale, derr.as<int>());
        M3R_CUDA(cudaEventRecord(ev.a, nullptr));
        for (int i = 0; i < it; ++i)
            m3r::attention_fwd(nullptr, dtype, dq.p, dk.p, dv.p, dout.p, n_seq, heads, nq, nk, scale, derr.as<int>());
        M3R_CUDA(cudaEventRecord(ev.b, nullptr));
        M3R_CUDA(cudaDeviceSynchronize());
        check_dev_err(derr.as<int>());
        if (kernel_ms) *kernel_ms = ev.ms() / it;
        M3R_CUDA(cudaMemcpy(out, dout.p, qn * 2, cudaMemcpyDeviceToHost));
    });
}

int m3r_gemm_test(int device, int dtype, const uint16_t* a, const uint16_t* w, const float* bias, float* c, int M,
                  int N, int K, int bn, int cta_pair, int iters, float* kernel_ms) {
    return guarded(nullptr, [&] {
        M3R_REQUIRE(a && w && c && M > 0 && N > 0 && K > 0 && K % 8 == 0 && N % 4 == 0, "gemm_test: bad arguments");
        m3r::DeviceGuard g(device);
        DBuf da(static_cast<size_t>(M) * K * 2), dw(static_cast<size_t>(N) * K * 2), dc(static_cast<size_t>(M) * N * 4),
            db(static_cast<size_t>(N) * 4), derr(sizeof(m3r::DevStatus));
        M3R_CUDA(cudaMemcpy(da.p, a, static_cast<size_t>(M) * K * 2, cudaMemcpyHostToDevice));
        M3R_CUDA(cudaMemcpy(dw.p, w, static_cast<size_t>(N) * K * 2, cudaMemcpyHostToDevice));
        if (bias) M3R_CUDA(cudaMemcpy(db.p, bias, static_cast<size_t>(N) * 4, cudaMemcpyHostToDevice));
        M3R_CUDA(cudaMemset(derr.p, 0, sizeof(m3r::DevStatus)));
        m3r::GemmParams p = m3r::gemm_params();
        p.bias = bias ? db.as<float>() : nullptr;
        p.out = dc.p;
        p.ldo = N;
        p.err = derr.as<int>();
        const int it = iters < 1 ? 1 : iters;
        Events ev;
        m3r::gemm_rows(nullptr, dtype, bn, m3r::EPI_F32, da.p, K, M, K, dw.p, K, N, p, cta_pair);
        M3R_CUDA(cudaEventRecord(ev.a, nullptr));
        for (int i = 0; i < it; ++i) m3r::gemm_rows(nullptr, dtype, bn, m3r::EPI_F32, da.p, K, M, K, dw.p, K, N, p, cta_pair);
        M3R_CUDA(cudaEventRecord(ev.b, nullptr));
        M3R_CUDA(cudaDeviceSynchronize());
        check_dev_err(derr.as<int>());
        if (kernel_ms) *kernel_ms = ev.ms() / it;
        M3R_CUDA(cudaMemcpy(c, dc.p, static_cast<size_t>(M) * N * 4, cudaMemcpyDeviceToHost));
    });
}

int m3r_gemm_resid_test(int device, int dtype, const uint16_t* a, const uint16_t* w, const float* bias, float* c,
                        int M, int N, int K, int bn, int cta_pair) {
    return guarded(nullptr, [&] {
        M3R_REQUIRE(a && w && c && M > 0 && N > 0 && K > 0 && K % 8 == 0 && N % 4 == 0,
                    "gemm_resid_test: bad arguments");
        m3r::DeviceGuard g(device);
        DBuf da(static_cast<size_t>(M) * K * 2), dw(static_cast<size_t>(N) * K * 2), dc(static_cast<size_t>(M) * N * 4),
            db(static_cast<size_t>(N) * 4), derr(sizeof(m3r::DevStatus));
        M3R_CUDA(cudaMemcpy(da.p, a, static_cast<size_t>(M) * K * 2, cudaMemcpyHostToDevice));
        M3R_CUDA(cudaMemcpy(dw.p, w, static_cast<size_t>(N) * K * 2, cudaMemcpyHostToDevice));
        M3R_CUDA(cudaMemcpy(dc.p, c, static_cast<size_t>(M) * N * 4, cudaMemcpyHostToDevice));
        if (bias) M3R_CUDA(cudaMemcpy(db.p, bias, static_cast<size_t>(N) * 4, cudaMemcpyHostToDevice));
        M3R_CUDA(cudaMemset(derr.p, 0, sizeof(m3r::DevStatus)));
        m3r::GemmParams p = m3r::gemm_params();
        p.bias = bias ? db.as<float>() : nullptr;
        p.out = dc.p;
        p.ldo = N;
        p.resid = dc.as<float>();
        p.ldr = N;
        p.err = derr.as<int>();
        m3r::gemm_rows(nullptr, dtype, bn, m3r::EPI_F32_RESID, da.p, K, M, K, dw.p, K, N, p, cta_pair);
        M3R_CUDA(cudaDeviceSynchronize());
        check_dev_err(derr.as<int>());
        M3R_CUDA(cudaMemcpy(c, dc.p, static_cast<size_t>(M) * N * 4, cudaMemcpyDeviceToHost));
    });
}

int m3r_conv3_test(int device, int dtype, const uint16_t* x, const uint16_t* w, const float* bias, float* y, int n,
                   int h, int wd, int c, int cout, int bn, int cta_pair) {
    return guarded(nullptr, [&] {
        M3R_REQUIRE(x && w && y && n > 0 && h > 0 && wd > 0 && c > 0 && c % 8 == 0 && cout > 0 && cout % 4 == 0,
                    "conv3_test: bad arguments");
        m3r::DeviceGuard g(device);
        const int cpad = (c + 63) / 64 * 64;
        const size_t xn = static_cast<size_t>(n) * h * wd * c, wn = static_cast<size_t>(cout) * 9 * cpad,
                     yn = static_cast<size_t>(n) * h * wd * cout;
        DBuf dx(xn * 2), dw(wn * 2), dy(yn * 4), db(static_cast<size_t>(cout) * 4), derr(sizeof(m3r::DevStatus));
        M3R_CUDA(cudaMemcpy(dx.p, x, xn * 2, cudaMemcpyHostToDevice));
        M3R_CUDA(cudaMemcpy(dw.p, w, wn * 2, cudaMemcpyHostToDevice));
        if (bias) M3R_CUDA(cudaMemcpy(db.p, bias, static_cast<size_t>(cout) * 4, cudaMemcpyHostToDevice));
        M3R_CUDA(cudaMemset(derr.p, 0, sizeof(m3r::DevStatus)));
        m3r::GemmParams p = m3r::gemm_params();
        p.bias = bias ? db.as<float>() : nullptr;
        p.out = dy.p;
        p.ldo = cout;
        p.err = derr.as<int>();
        m3r::gemm_conv3(nullptr, dtype, bn, m3r::EPI_F32, dx.p, n, h, wd, c, c, dw.p, cout, p, cta_pair);
        M3R_CUDA(cudaDeviceSynchronize());
        check_dev_err(derr.as<int>());
        M3R_CUDA(cudaMemcpy(y, dy.p, yn * 4, cudaMemcpyDeviceToHost));
    });
}

int m3r_match_nn(int device, const float* desc_1, const float* desc_2, int64_t n1, int64_t n2, int desc_dim,
                 int32_t* nn_12, int32_t* nn_21, float* best_12, float* kernel_ms) {
    return guarded(nullptr, [&] {
        M3R_REQUIRE(desc_1 && desc_2 && nn_12 && nn_21 && n1 > 0 && n2 > 0 && desc_dim > 0 && n1 < 0x7FFFFFFF &&
                        n2 < 0x7FFFFFFF,
                    "match_nn: bad arguments");
        m3r::DeviceGuard g(device);
        DBuf a(static_cast<size_t>(n1) * desc_dim * 4), b(static_cast<size_t>(n2) * desc_dim * 4), rk(n1 * 8),
            ck(n2 * 8), i12(n1 * 4), i21(n2 * 4);
        M3R_CUDA(cudaMemcpy(a.p, desc_1, static_cast<size_t>(n1) * desc_dim * 4, cudaMemcpyHostToDevice));
        M3R_CUDA(cudaMemcpy(b.p, desc_2, static_cast<size_t>(n2) * desc_dim * 4, cudaMemcpyHostToDevice));
        Events ev;
        m3r::match_normalize(nullptr, a.as<float>(), a.as<float>(), n1, desc_dim);
        m3r::match_normalize(nullptr, b.as<float>(), b.as<float>(), n2, desc_dim);
        M3R_CUDA(cudaEventRecord(ev.a, nullptr));
        m3r::match_argmax(nullptr, a.as<float>(), b.as<float>(), 0, n1, n2, desc_dim, rk.as<unsigned long long>(),
                          ck.as<unsigned long long>(), true);
        M3R_CUDA(cudaEventRecord(ev.b, nullptr));
        m3r::match_decode(nullptr, rk.as<unsigned long long>(), n1, i12.as<int32_t>());
        m3r::match_decode(nullptr, ck.as<unsigned long long>(), n2, i21.as<int32_t>());
        M3R_CUDA(cudaDeviceSynchronize());
        if (kernel_ms) *kernel_ms = ev.ms();
        M3R_CUDA(cudaMemcpy(nn_12, i12.p, n1 * 4, cudaMemcpyDeviceToHost));
        M3R_CUDA(cudaMemcpy(nn_21, i21.p, n2 * 4, cudaMemcpyDeviceToHost));
        if (best_12) {
            std::vector<unsigned long long> keys(static_cast<size_t>(n1));
            M3R_CUDA(cudaMemcpy(keys.data(), rk.p, n1 * 8, cudaMemcpyDeviceToHost));
            for (int64_t i = 0; i < n1; ++i) {
                const uint32_t k = static_cast<uint32_t>(keys[i] >> 32);
                const uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
                float f;
                std::memcpy(&f, &u, 4);
                best_12[i] = f;
            }
        }
    });
}

}  // extern "C"
