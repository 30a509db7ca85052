// Two-view forward pass on one device and its multi-device orchestration.
//
// Token layout: all 2n images of a launch (view 1 pairs 0..n-1, then view 2
// pairs 0..n-1) are rows of one [2n * N, D] activation matrix, so the shared-
// weight encoder runs as single GEMMs over every token.  The decoder runs per
// view (different weights, dec_blocks / dec_blocks2), each view's rows being a
// contiguous half.  Residual streams stay fp32; GEMM operands are 16-bit (fp16 or
// bf16, Dims::dt) with fp32 accumulation.
//
// Reference semantics: encoder croco_encoder.py:245-283, decoder
// croco_decoder.py:395-434, heads mpsgraph_engine.mm:383-437 (see oracle/model.py
// for the restatement the tests check against).
#include "engine.h"

#include <algorithm>
#include <cstddef>
#include <array>
#include <map>
#include <mutex>
#include <cstdio>
#include <chrono>
#include <cmath>
#include <cstring>
#include <functional>
#include <thread>

#include "attention.h"
#include "common.cuh"
#include "gemm.h"
#include "kernels.h"
#include "nccl_dl.h"
#include "safetensors.h"

namespace m3r {

// ---------------------------------------------------------------------------- dims
Dims Dims::from(const m3r_config& c) {
    Dims d;
    d.patch = c.patch;
    d.enc_dim = c.enc_dim;
    d.enc_depth = c.enc_depth;
    d.enc_heads = c.enc_heads;
    d.enc_mlp = c.enc_mlp;
    d.dec_dim = c.dec_dim;
    d.dec_depth = c.dec_depth;
    d.dec_heads = c.dec_heads;
    d.dec_mlp = c.dec_mlp;
    d.lf_hidden = c.lf_hidden;
    d.desc_dim = c.desc_dim;
    d.head = c.head;
    d.H = c.img_h;
    d.W = c.img_w;
    M3R_REQUIRE(d.patch > 0 && d.H > 0 && d.W > 0 && d.H % d.patch == 0 && d.W % d.patch == 0,
                "image size must be a positive multiple of the patch size");
    d.hg = d.H / d.patch;
    d.wg = d.W / d.patch;
    d.ntok = d.hg * d.wg;
    d.kpad = (3 * d.patch * d.patch + 63) / 64 * 64;
    d.hook1 = d.dec_depth / 2 - 1;
    d.hook2 = d.dec_depth * 3 / 4 - 1;
    d.dt = c.dtype;
    M3R_REQUIRE(d.dt == DT_F16 || d.dt == DT_BF16, "dtype must be M3R_DTYPE_F16 or M3R_DTYPE_BF16");
    d.dpt_h = 16 * d.hg;
    d.dpt_w = 16 * d.wg;
    M3R_REQUIRE(d.enc_heads > 0 && d.enc_dim == 64 * d.enc_heads, "encoder head dim must be 64");
    M3R_REQUIRE(d.dec_heads > 0 && d.dec_dim == 64 * d.dec_heads, "decoder head dim must be 64");
    M3R_REQUIRE(d.enc_dim % 128 == 0 && d.dec_dim % 128 == 0, "model dims must be multiples of 128");
    M3R_REQUIRE(d.enc_mlp % 64 == 0 && d.dec_mlp % 64 == 0 && d.lf_hidden % 64 == 0, "MLP widths must be multiples of 64");
    M3R_REQUIRE(d.enc_dim <= 1024 && d.dec_dim <= 1024, "model dims above 1024 are not supported");
    M3R_REQUIRE(d.head == M3R_HEAD_MAST3R24 || d.head == M3R_HEAD_REF_SIMPLE, "unknown head");
    M3R_REQUIRE(d.desc_dim == (d.head == M3R_HEAD_MAST3R24 ? 24 : 256),
                "descriptor dim must be 24 (MASt3R head) or 256 (reference CPU head)");
    M3R_REQUIRE((d.patch * d.patch) % 8 == 0 || (d.patch * d.patch) % 4 == 0, "unsupported patch size");
    M3R_REQUIRE(d.hg % 2 == 0 && d.wg % 2 == 0, "patch grid must have even height and width");
    M3R_REQUIRE(d.dec_depth >= 4, "decoder depth must be >= 4");
    return d;
}

DeviceGuard::DeviceGuard(int dev) {
    M3R_CUDA(cudaGetDevice(&prev));
    M3R_CUDA(cudaSetDevice(dev));
}
DeviceGuard::~DeviceGuard() { cudaSetDevice(prev); }

// ---------------------------------------------------------------------------- host weight prep
namespace {

// float -> 16-bit operand bits, round to nearest even (CUDA's host-side conversions)
uint16_t to16bits(float f, int dt) {
    uint16_t r;
    if (dt == DT_F16) {
        const __half h = __float2half_rn(f);
        std::memcpy(&r, &h, 2);
    } else {
        const __nv_bfloat16 h = __float2bfloat16_rn(f);
        std::memcpy(&r, &h, 2);
    }
    return r;
}

// memcpy split over host threads (large copies between pinned staging and pageable
// caller memory run at several times one thread's bandwidth)
void parallel_memcpy(void* dst, const void* src, size_t n) {
    constexpr size_t kChunk = size_t(16) << 20;
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    const size_t nt = std::min<size_t>(std::min<size_t>(8, hw), (n + kChunk - 1) / kChunk);
    if (nt <= 1) {
        std::memcpy(dst, src, n);
        return;
    }
    std::vector<std::thread> th;
    const size_t per = (n + nt - 1) / nt;
    for (size_t t = 0; t < nt; ++t) {
        const size_t b = t * per, e = std::min(n, b + per);
        if (b >= e) break;
        th.emplace_back([=] { std::memcpy(static_cast<char*>(dst) + b, static_cast<const char*>(src) + b, e - b); });
    }
    for (auto& x : th) x.join();
}

struct HostLin {
    std::vector<uint16_t> w;  // 16-bit operand bits [out, in]
    std::vector<float> b;     // may be empty
    int out = 0, in = 0;
};

HostLin to16(int dt, const std::vector<float>& w, int out, int in, std::vector<float> b = {}) {
    HostLin h;
    h.out = out;
    h.in = in;
    h.w.resize(static_cast<size_t>(out) * in);
    for (size_t i = 0; i < h.w.size(); ++i) h.w[i] = to16bits(w[i], dt);
    h.b = std::move(b);
    return h;
}

// conv weight [co, ci, 3, 3] -> [co, 9, cpad] tap-major, zero channel padding
HostLin conv3_weights(int dt, const std::vector<float>& w, int co, int ci, std::vector<float> b = {}) {
    const int cpad = (ci + 63) / 64 * 64;
    std::vector<float> t(static_cast<size_t>(co) * 9 * cpad, 0.0f);
    for (int o = 0; o < co; ++o)
        for (int c = 0; c < ci; ++c)
            for (int tap = 0; tap < 9; ++tap)
                t[(static_cast<size_t>(o) * 9 + tap) * cpad + c] = w[(static_cast<size_t>(o) * ci + c) * 9 + tap];
    return to16(dt, t, co, 9 * cpad, std::move(b));
}

// ConvTranspose2d weight [ci, co, s, s] -> B [(dy*s+dx)*co + o, ci]
HostLin convt_weights(int dt, const std::vector<float>& w, int ci, int co, int s, std::vector<float> b) {
    std::vector<float> t(static_cast<size_t>(s) * s * co * ci);
    for (int c = 0; c < ci; ++c)
        for (int o = 0; o < co; ++o)
            for (int dy = 0; dy < s; ++dy)
                for (int dx = 0; dx < s; ++dx)
                    t[(static_cast<size_t>((dy * s + dx) * co + o)) * ci + c] =
                        w[((static_cast<size_t>(c) * co + o) * s + dy) * s + dx];
    return to16(dt, t, s * s * co, ci, std::move(b));
}

}  // namespace

// ---------------------------------------------------------------------------- device
class Device {
public:
    Device(int dev, const Dims& d, int max_pairs) : dev_(dev), d_(d), max_pairs_(max_pairs) {
        DeviceGuard g(dev_);
        M3R_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
        M3R_CUDA(cudaStreamCreateWithFlags(&copy_stream_, cudaStreamNonBlocking));
        err_ = static_cast<int*>(alloc(sizeof(DevStatus)));
        M3R_CUDA(cudaMemset(err_, 0, sizeof(DevStatus)));
        for (int i = 0; i < 8; ++i) M3R_CUDA(cudaEventCreate(&stage_ev_[i]));
        alloc_activations();
    }
    ~Device() {
        cudaSetDevice(dev_);
        if (stream_) cudaStreamSynchronize(stream_);
        for (auto& g : graphs_)
            for (cudaGraphExec_t e : g.second)
                if (e) cudaGraphExecDestroy(e);
        for (auto& e : prof_ev_) cudaEventDestroy(e);
        for (int i = 0; i < 8; ++i) cudaEventDestroy(stage_ev_[i]);
        for (auto& e : chunk_ev_) cudaEventDestroy(e);
        if (copy_stream_) {
            cudaStreamSynchronize(copy_stream_);
            cudaStreamDestroy(copy_stream_);
        }
        for (void* p : allocs_) cudaFree(p);
        if (stream_) cudaStreamDestroy(stream_);
        for (void* p : {stage_in_, stage_out_[0], stage_out_[1]})
            if (p) cudaFreeHost(p);
        if (raw_) cudaFree(raw_);
    }

    int dev() const { return dev_; }
    cudaStream_t stream() const { return stream_; }

    void* alloc(size_t bytes) {
        void* p = nullptr;
        M3R_CUDA(cudaMalloc(&p, bytes > 0 ? bytes : 16));
        allocs_.push_back(p);
        return p;
    }
    template <class T>
    T* upload(const std::vector<T>& v) {
        if (v.empty()) return nullptr;
        T* p = static_cast<T*>(alloc(v.size() * sizeof(T)));
        M3R_CUDA(cudaMemcpy(p, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice));
        return p;
    }
    Lin upload(const HostLin& h) {
        Lin l;
        l.out = h.out;
        l.in = h.in;
        l.w = upload(h.w);
        l.b = upload(h.b);
        return l;
    }
    Norm upload_norm(const std::vector<float>& g, const std::vector<float>& b) { return Norm{upload(g), upload(b)}; }

    // ------------------------------------------------------------ weights (filled by Engine::load)
    Lin patch;
    std::vector<EncBlock> enc;
    Norm enc_norm;
    Lin dec_embed;
    std::vector<DecBlock> dec[2];
    Norm dec_norm;
    Norm unit_norm;  // gamma 1, beta 0 (decoder width): norm_y without its affine part
    Head head[2];
    float* rope_cos = nullptr;
    float* rope_sin = nullptr;
    Lin whiten;               // retrieval whitening: W = P^T [D, D], bias = -(m P) (Engine::load_retrieval)
    float* rattn = nullptr;   // retrieval attention weights [2 * max_pairs * N]

    // ------------------------------------------------------------ activations
    uint8_t* img = nullptr;
    uint16_t *patches = nullptr, *xn = nullptr, *yn = nullptr, *q = nullptr, *k = nullptr, *v = nullptr,
                  *ao = nullptr, *h = nullptr, *enc_out = nullptr, *hook1 = nullptr, *hook2 = nullptr,
                  *dec_out = nullptr;
    float *xenc = nullptr, *xdec = nullptr, *encp = nullptr;
    uint16_t *f0a = nullptr, *f0 = nullptr, *rn0 = nullptr, *f1a = nullptr, *f1 = nullptr, *rn1 = nullptr,
                  *f2 = nullptr, *rn2 = nullptr, *f3a = nullptr, *col3 = nullptr, *f3 = nullptr, *rn3 = nullptr,
                  *fused = nullptr, *up1 = nullptr, *hd0 = nullptr, *up2 = nullptr, *lf1 = nullptr;
    float* out4 = nullptr;
    uint16_t* hdg = nullptr;  // reference CPU head: first conv's output at grid resolution
    float* rawd = nullptr;    // reference CPU head: first 256 local-feature channels [tokens, 256]
    float *o_pts = nullptr, *o_conf = nullptr, *o_desc = nullptr;
    MatchWorkspace mws;

    int staged = 0;  // pairs staged on this device

    void alloc_activations() {
        const long long P = max_pairs_;
        const long long T = 2 * P * d_.ntok, Tv = P * d_.ntok;
        const long long Dm = std::max(d_.enc_dim, d_.dec_dim);
        const long long Hm = std::max(d_.enc_mlp, d_.dec_mlp);
        const long long hg = d_.hg, wg = d_.wg;
        auto bf = [&](long long n) { return static_cast<uint16_t*>(alloc(n * 2)); };
        auto f32 = [&](long long n) { return static_cast<float*>(alloc(n * 4)); };
        img = static_cast<uint8_t*>(alloc(2 * P * d_.H * d_.W * 3));
        patches = bf(T * d_.kpad);
        xenc = f32(T * d_.enc_dim);
        xdec = f32(T * d_.dec_dim);
        encp = f32(T * d_.dec_dim);
        xn = bf(T * Dm);
        yn = bf(T * Dm);
        q = bf(T * Dm);
        k = bf(T * Dm);
        v = bf(T * Dm);
        ao = bf(T * Dm);
        h = bf(T * Hm);
        enc_out = bf(T * d_.enc_dim);
        hook1 = bf(T * d_.dec_dim);
        hook2 = bf(T * d_.dec_dim);
        dec_out = bf(T * d_.dec_dim);
        rattn = f32(T);
        lf1 = bf(Tv * d_.lf_hidden);
        o_pts = f32(2 * P * d_.H * d_.W * 3);
        o_conf = f32(2 * P * d_.H * d_.W);
        o_desc = f32(2 * P * d_.H * d_.W * d_.desc_dim);
        if (d_.head == M3R_HEAD_REF_SIMPLE) {
            // the reference CPU head works at patch-grid resolution, one view at a time
            hdg = bf(Tv * 128);
            out4 = f32(Tv * 4);
            rawd = f32(Tv * 256);
            return;
        }
        // DPT / local features, one view at a time
        f0a = bf(Tv * 96);
        f0 = bf(P * 16 * hg * wg * 96);
        rn0 = bf(P * 16 * hg * wg * 256);
        f1a = bf(Tv * 192);
        f1 = bf(P * 4 * hg * wg * 192);
        rn1 = bf(P * 4 * hg * wg * 256);
        f2 = bf(Tv * 384);
        rn2 = bf(P * hg * wg * 256);
        f3a = bf(Tv * 768);
        col3 = bf(P * (hg / 2) * (wg / 2) * 9 * 768);
        f3 = bf(P * (hg / 2) * (wg / 2) * 768);
        rn3 = bf(P * (hg / 2) * (wg / 2) * 256);
        fused = bf(P * 16 * hg * wg * 256);
        up1 = bf(P * 64 * hg * wg * 256);
        hd0 = bf(P * 64 * hg * wg * 128);
        up2 = bf(P * 256 * hg * wg * 128);
        out4 = f32(P * 256 * hg * wg * 4);
    }

    // ------------------------------------------------------------ profiling
    struct Prof {
        double ms[3] = {0, 0, 0};
        double flops[3] = {0, 0, 0};
        long launches[3] = {0, 0, 0};
    } prof;
    bool profiling = false;
    std::vector<cudaEvent_t> prof_ev_;
    struct ProfRec {
        int cat;
        double flops;
        const char* op;
    };
    std::vector<ProfRec> prof_rec_;  // per event pair
    struct OpStat {
        std::string op;
        double ms = 0, flops = 0;
        long launches = 0;
    };
    std::vector<OpStat> prof_ops;  // per operation of the model, in order of first launch

    template <class F>
    void launch(int cat, double flops, const char* op, F&& fn) {
        if (!profiling) {
            fn();
            return;
        }
        const size_t i = prof_rec_.size();
        while (prof_ev_.size() < 2 * (i + 1)) {
            cudaEvent_t e;
            M3R_CUDA(cudaEventCreate(&e));
            prof_ev_.push_back(e);
        }
        M3R_CUDA(cudaEventRecord(prof_ev_[2 * i], stream_));
        fn();
        M3R_CUDA(cudaEventRecord(prof_ev_[2 * i + 1], stream_));
        prof_rec_.push_back({cat, flops, op});
    }
    void collect_profile() {
        prof = Prof();
        prof_ops.clear();
        for (size_t i = 0; i < prof_rec_.size(); ++i) {
            float ms = 0;
            M3R_CUDA(cudaEventElapsedTime(&ms, prof_ev_[2 * i], prof_ev_[2 * i + 1]));
            const ProfRec& r = prof_rec_[i];
            prof.ms[r.cat] += ms;
            prof.flops[r.cat] += r.flops;
            prof.launches[r.cat] += 1;
            OpStat* st = nullptr;
            for (auto& o : prof_ops)
                if (o.op == r.op) st = &o;
            if (st == nullptr) {
                prof_ops.push_back(OpStat{r.op});
                st = &prof_ops.back();
            }
            st->ms += ms;
            st->flops += r.flops;
            st->launches += 1;
        }
        prof_rec_.clear();
    }

    // ------------------------------------------------------------ building blocks
    static constexpr int kGemm = 0, kAttn = 1, kOther = 2;

    int bn_for(int n) const { return (n % 256 == 0) ? 256 : 128; }

    GemmParams gp() const {
        GemmParams p = gemm_params();
        p.err = err_;
        return p;
    }

    void linear(const char* op, const uint16_t* A, long long M, const Lin& L, int epi, void* out, long long ldo,
                int act = ACT_NONE, const float* resid = nullptr, int bn = 0) {
        GemmParams p = gp();
        p.bias = L.b;
        p.act = act;
        p.out = out;
        p.ldo = ldo;
        p.resid = resid;
        p.ldr = ldo;
        const int b = bn ? bn : bn_for(L.out);
        launch(kGemm, 2.0 * M * L.out * L.in, op,
               [&] { gemm_rows(stream_, d_.dt, b, epi, A, L.in, static_cast<int>(M), L.in, L.w, L.in, L.out, p); });
    }

    // head-major scatter of [M, nsec * D] into up to three [seqs, heads, ntok, 64] buffers
    void linear_heads(const char* op, const uint16_t* A, long long M, const Lin& L, int D, uint16_t* o0, int r0,
                      uint16_t* o1, int r1, uint16_t* o2, int r2) {
        GemmParams p = gp();
        p.bias = L.b;
        p.sec_len = D;
        p.n_tok = d_.ntok;
        p.grid_w = d_.wg;
        p.sec_out[0] = o0;
        p.sec_out[1] = o1;
        p.sec_out[2] = o2;
        p.sec_rope[0] = r0;
        p.sec_rope[1] = r1;
        p.sec_rope[2] = r2;
        p.rope_cos = rope_cos;
        p.rope_sin = rope_sin;
        p.rope_npos = std::max(d_.hg, d_.wg);
        const int b = (D % 256 == 0) ? 256 : 128;
        launch(kGemm, 2.0 * M * L.out * L.in, op,
               [&] { gemm_rows(stream_, d_.dt, b, EPI_HEADS, A, L.in, static_cast<int>(M), L.in, L.w, L.in, L.out, p); });
    }

    void attn(const char* op, const uint16_t* qq, const uint16_t* kk, const uint16_t* vv, uint16_t* out, int seqs,
              int heads) {
        const double fl = 4.0 * seqs * heads * static_cast<double>(d_.ntok) * d_.ntok * 64;
        launch(kAttn, fl, op, [&] { attention_fwd(stream_, d_.dt, qq, kk, vv, out, seqs, heads, d_.ntok, d_.ntok, 0.125f, err_); });
    }

    void ln(const char* op, const float* x, long long rows, int D, const Norm& n, uint16_t* y) {
        launch(kOther, 0, op, [&] { layernorm(stream_, d_.dt, x, static_cast<int>(rows), D, n.g, n.b, y); });
    }

    void conv3(const char* op, const uint16_t* X, int n, int hh, int ww, int c, const Lin& L, int epi, void* out, int act,
               int bn, const float* w4 = nullptr, const float* b4 = nullptr) {
        GemmParams p = gp();
        p.bias = L.b;
        p.act = act;
        p.out = out;
        p.ldo = L.out;
        p.w4 = w4;
        p.b4 = b4;
        const double fl = 2.0 * n * hh * ww * static_cast<double>(L.out) * 9 * c;
        launch(kGemm, fl, op, [&] { gemm_conv3(stream_, d_.dt, bn, epi, X, n, hh, ww, c, c, L.w, L.out, p); });
    }

    // ------------------------------------------------------------ forward
    // One forward pass over n pairs whose images sit in input slots [slot, slot + n)
    // and whose outputs go to output slots [slot, slot + n), in four stages (patch
    // embedding, encoder, decoder, heads) with a timing event (ev[0..4]) before and
    // after each.  The first pass for a given (n, slot) launches directly (it also sets
    // the kernels' attributes); later passes replay one CUDA graph per stage, captured
    // on the second pass.  Only the patch stage (reads the input slot) and the heads
    // (write the output slot) depend on the slot: the encoder and decoder graphs are
    // shared by every slot of a pair count.  Profiled passes always launch directly
    // (events around every launch).  enqueue_forward only enqueues; forward also waits
    // and reads the timings.
    static constexpr int kStages = 4;
    void enqueue_forward(int n, int slot, const cudaEvent_t* ev) {
        DeviceGuard g(dev_);
        profiling_reset();
        const std::pair<int, int> key(n, slot);
        const bool use_graph = !profiling && direct_runs_[key]++ > 0;
        M3R_CUDA(cudaEventRecord(ev[0], stream_));
        for (int st = 0; st < kStages; ++st) {
            if (!use_graph) {
                enqueue_stage(st, n, slot);
            } else {
                const bool slotted = st == 0 || st == kStages - 1;
                cudaGraphExec_t& ge = graphs_[std::make_pair(n, slotted ? slot : -1)][st];
                if (ge == nullptr) ge = capture_stage(st, n, slot);
                M3R_CUDA(cudaGraphLaunch(ge, stream_));
            }
            M3R_CUDA(cudaEventRecord(ev[st + 1], stream_));
        }
    }

    // stage_ms[0..3] per stage, stage_ms[4] whole pass, from events ev[0..4]
    static void stage_times(const cudaEvent_t* ev, float* stage_ms) {
        float ms;
        for (int i = 0; i < kStages; ++i) {
            M3R_CUDA(cudaEventElapsedTime(&ms, ev[i], ev[i + 1]));
            stage_ms[i] = ms;
        }
        M3R_CUDA(cudaEventElapsedTime(&ms, ev[0], ev[kStages]));
        stage_ms[kStages] = ms;
    }

    void forward(int n, float* stage_ms) {
        enqueue_forward(n, 0, stage_ev_);
        M3R_CUDA(cudaStreamSynchronize(stream_));
        check_error();
        if (profiling) collect_profile();
        if (stage_ms) stage_times(stage_ev_, stage_ms);
    }

    cudaGraphExec_t capture_stage(int st, int n, int slot) {
        cudaGraph_t graph = nullptr;
        M3R_CUDA(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
        try {
            enqueue_stage(st, n, slot);
        } catch (...) {
            cudaStreamEndCapture(stream_, &graph);
            if (graph) cudaGraphDestroy(graph);
            throw;
        }
        M3R_CUDA(cudaStreamEndCapture(stream_, &graph));
        cudaGraphExec_t exec = nullptr;
        const cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        M3R_CUDA(e);
        return exec;
    }

    // Slot layout of the inputs and outputs: view v of the pair in slot s is image /
    // output v * max_pairs + s, so sub-batches in different slots never overlap.
    uint8_t* img_slot(int view, int slot) const {
        return img + (static_cast<size_t>(view) * max_pairs_ + slot) * d_.H * d_.W * 3;
    }
    float* out_slot(const float* base, int per_pixel, int view, int slot) const {
        return const_cast<float*>(base) + (static_cast<size_t>(view) * max_pairs_ + slot) * d_.H * d_.W * per_pixel;
    }

    // Enqueues every launch of stage st of one forward pass on the device's stream.
    void enqueue_stage(int st, int n, int slot) {
        switch (st) {
            case 0: stage_patch(n, slot); break;
            case 1: stage_encoder(n); break;
            case 2: stage_decoder(n); break;
            default:
                // heads, one view at a time (downstream_head1 / downstream_head2)
                for (int view = 0; view < 2; ++view) {
                    if (d_.head == M3R_HEAD_REF_SIMPLE)
                        heads_ref(view, n, slot);
                    else
                        heads(view, n, slot);
                }
        }
    }

    // patch embedding (+ ImageNet normalisation fused into the im2col)
    void stage_patch(int n, int slot) {
        const Dims& d = d_;
        const long long T = 2LL * n * d.ntok;
        launch(kOther, 0, "patch.im2col", [&] {
            patch_im2col(stream_, d_.dt, img_slot(0, slot), img_slot(1, slot), n, 2 * n, d.H, d.W, d.patch, d.kpad,
                         patches);
        });
        GemmParams p = gp();
        p.bias = patch.b;
        p.out = xenc;
        p.ldo = d.enc_dim;
        launch(kGemm, 2.0 * T * d.enc_dim * 3 * d.patch * d.patch, "patch.gemm", [&] {
            gemm_rows(stream_, d_.dt, bn_for(d.enc_dim), EPI_F32, patches, d.kpad, static_cast<int>(T), d.kpad,
                      patch.w, d.kpad, d.enc_dim, p);
        });
    }

    // encoder (croco_encoder.py:142-168), both views of every pair in one pass
    void stage_encoder(int n) {
        const Dims& d = d_;
        const long long T = 2LL * n * d.ntok;
        const int De = d.enc_dim;
        for (int i = 0; i < d.enc_depth; ++i) {
            const EncBlock& B = enc[i];
            ln("enc.ln", xenc, T, De, B.n1, xn);
            linear_heads("enc.qkv", xn, T, B.qkv, De, q, 1, k, 1, v, 0);
            attn("enc.attn", q, k, v, ao, 2 * n, d.enc_heads);
            linear("enc.proj", ao, T, B.proj, EPI_F32_RESID, xenc, De, ACT_NONE, xenc);
            ln("enc.ln", xenc, T, De, B.n2, xn);
            linear("enc.fc1", xn, T, B.fc1, EPI_BF16, h, d.enc_mlp, ACT_GELU);
            linear("enc.fc2", h, T, B.fc2, EPI_F32_RESID, xenc, De, ACT_NONE, xenc);
        }
        ln("enc.ln", xenc, T, De, enc_norm, enc_out);
    }

    // decoder (croco_decoder.py:395-434)
    void stage_decoder(int n) {
        const Dims& d = d_;
        const long long T = 2LL * n * d.ntok;
        const long long Tv = static_cast<long long>(n) * d.ntok;
        const int Dd = d.dec_dim;
        linear("dec.embed", enc_out, T, dec_embed, EPI_F32, encp, Dd);
        M3R_CUDA(cudaMemcpyAsync(xdec, encp, sizeof(float) * T * Dd, cudaMemcpyDeviceToDevice, stream_));
        // normalised projected encoder output of both views (norm_y's affine part lives
        // in the K/V projection weights)
        ln("dec.ln", encp, T, Dd, unit_norm, yn);
        // The two views' blocks are independent within a block (the cross attention reads
        // the other view's projected encoder output, constant over blocks), so each
        // attention runs once over both views' 2n sequences; the projections and MLPs
        // keep their per-view weights (dec_blocks / dec_blocks2).  View v's sequences,
        // tokens and head-major Q/K/V planes start at v * Tv rows.
        auto xv = [&](int view) { return xdec + view * Tv * Dd; };
        auto xnv = [&](int view) { return xn + view * Tv * Dd; };
        auto aov = [&](int view) { return ao + view * Tv * Dd; };
        auto qv = [&](uint16_t* base, int view) { return base + view * Tv * Dd; };
        for (int i = 0; i < d.dec_depth; ++i) {
            // self attention
            for (int view = 0; view < 2; ++view) {
                const DecBlock& B = dec[view][i];
                ln("dec.ln", xv(view), Tv, Dd, B.n1, xnv(view));
                linear_heads("dec.qkv", xnv(view), Tv, B.qkv, Dd, qv(q, view), 1, qv(k, view), 1, qv(v, view), 0);
            }
            attn("dec.attn_self", q, k, v, ao, 2 * n, d.dec_heads);
            for (int view = 0; view < 2; ++view)
                linear("dec.proj", aov(view), Tv, dec[view][i].proj, EPI_F32_RESID, xv(view), Dd, ACT_NONE, xv(view));
            // cross attention: queries from this view, keys/values from the other view's
            // projected encoder output
            for (int view = 0; view < 2; ++view) {
                const DecBlock& B = dec[view][i];
                const uint16_t* yno = yn + (1 - view) * Tv * Dd;  // the other view
                ln("dec.ln", xv(view), Tv, Dd, B.n2, xnv(view));
                linear_heads("dec.q", xnv(view), Tv, B.q, Dd, qv(q, view), 1, nullptr, 0, nullptr, 0);
                linear_heads("dec.kv", yno, Tv, B.kv, Dd, qv(k, view), 1, qv(v, view), 0, nullptr, 0);
            }
            attn("dec.attn_cross", q, k, v, ao, 2 * n, d.dec_heads);
            for (int view = 0; view < 2; ++view) {
                const DecBlock& B = dec[view][i];
                linear("dec.cproj", aov(view), Tv, B.cproj, EPI_F32_RESID, xv(view), Dd, ACT_NONE, xv(view));
                // MLP
                ln("dec.ln", xv(view), Tv, Dd, B.n3, xnv(view));
                linear("dec.fc1", xnv(view), Tv, B.fc1, EPI_BF16, h, d.dec_mlp, ACT_GELU);
                linear("dec.fc2", h, Tv, B.fc2, EPI_F32_RESID, xv(view), Dd, ACT_NONE, xv(view));
            }
            if (i == d.hook1) launch(kOther, 0, "dec.hook_cast", [&] { cast16(stream_, d_.dt, xdec, T * Dd, hook1); });
            if (i == d.hook2) launch(kOther, 0, "dec.hook_cast", [&] { cast16(stream_, d_.dt, xdec, T * Dd, hook2); });
        }
        ln("dec.ln", xdec, T, Dd, dec_norm, dec_out);
    }

    void heads(int view, int n, int slot) {
        const Dims& d = d_;
        const Head& Hh = head[view];
        const long long N = d.ntok, Tv = static_cast<long long>(n) * N;
        const int hg = d.hg, wg = d.wg;
        const uint16_t* h0 = enc_out + view * Tv * d.enc_dim;
        const uint16_t* h1 = hook1 + view * Tv * d.dec_dim;
        const uint16_t* h2 = hook2 + view * Tv * d.dec_dim;
        const uint16_t* h3 = dec_out + view * Tv * d.dec_dim;

        // act_postprocess (mpsgraph_engine.mm:391-395)
        linear("head.act_post", h0, Tv, Hh.ap0_0, EPI_BF16, f0a, 96, ACT_NONE, nullptr, 128);
        {
            GemmParams p = gp();
            p.bias = Hh.ap0_1t.b;
            p.out = f0;
            p.ldo = 96;
            p.ct_s = 4;
            p.ct_cout = 96;
            p.ct_h = hg;
            p.ct_w = wg;
            launch(kGemm, 2.0 * Tv * Hh.ap0_1t.out * Hh.ap0_1t.in, "head.convT",
                   [&] { gemm_rows(stream_, d_.dt, 256, EPI_CONVT, f0a, 96, static_cast<int>(Tv), 96, Hh.ap0_1t.w, 96, Hh.ap0_1t.out, p); });
        }
        linear("head.act_post", h1, Tv, Hh.ap1_0, EPI_BF16, f1a, 192, ACT_NONE, nullptr, 128);
        {
            GemmParams p = gp();
            p.bias = Hh.ap1_1t.b;
            p.out = f1;
            p.ldo = 192;
            p.ct_s = 2;
            p.ct_cout = 192;
            p.ct_h = hg;
            p.ct_w = wg;
            launch(kGemm, 2.0 * Tv * Hh.ap1_1t.out * Hh.ap1_1t.in, "head.convT",
                   [&] { gemm_rows(stream_, d_.dt, 256, EPI_CONVT, f1a, 192, static_cast<int>(Tv), 192, Hh.ap1_1t.w, 192, Hh.ap1_1t.out, p); });
        }
        linear("head.act_post", h2, Tv, Hh.ap2_0, EPI_BF16, f2, 384, ACT_NONE, nullptr, 128);
        linear("head.act_post", h3, Tv, Hh.ap3_0, EPI_BF16, f3a, 768, ACT_NONE, nullptr, 256);
        launch(kOther, 0, "head.im2col", [&] { im2col_s2(stream_, f3a, n, hg, wg, 768, col3); });
        linear("head.act_post", col3, static_cast<long long>(n) * (hg / 2) * (wg / 2), Hh.ap3_1, EPI_BF16, f3, 768, ACT_NONE, nullptr, 256);

        // layer_rn (3x3, no bias) -> 256 channels each
        conv3("head.layer_rn", f0, n, 4 * hg, 4 * wg, 96, Hh.rn[0], EPI_BF16, rn0, ACT_NONE, 256);
        conv3("head.layer_rn", f1, n, 2 * hg, 2 * wg, 192, Hh.rn[1], EPI_BF16, rn1, ACT_NONE, 256);
        conv3("head.layer_rn", f2, n, hg, wg, 384, Hh.rn[2], EPI_BF16, rn2, ACT_NONE, 256);
        conv3("head.layer_rn", f3, n, hg / 2, wg / 2, 768, Hh.rn[3], EPI_BF16, rn3, ACT_NONE, 256);

        // fusion and head (graph_builder.hpp:285-299, mpsgraph_engine.mm:402-422)
        const int H0 = 4 * hg, W0 = 4 * wg;
        launch(kOther, 0, "head.fuse", [&] { dpt_fuse(stream_, d_.dt, rn0, rn1, 2 * hg, 2 * wg, rn2, hg, wg, rn3, hg / 2, wg / 2, n, H0, W0, 256, fused); });
        launch(kOther, 0, "head.resize", [&] { resize16(stream_, d_.dt, fused, n, H0, W0, 256, 2 * H0, 2 * W0, up1); });
        conv3("head.conv0", up1, n, 2 * H0, 2 * W0, 256, Hh.hd0, EPI_BF16, hd0, ACT_RELU, 128);
        launch(kOther, 0, "head.resize", [&] { resize16(stream_, d_.dt, hd0, n, 2 * H0, 2 * W0, 128, 4 * H0, 4 * W0, up2); });
        conv3("head.conv_out", up2, n, 4 * H0, 4 * W0, 128, Hh.hd2, EPI_HEAD4, out4, ACT_RELU, 128, Hh.w4, Hh.b4);
        float* pts = out_slot(o_pts, 3, view, slot);
        float* conf = out_slot(o_conf, 1, view, slot);
        launch(kOther, 0, "head.split", [&] { head_split(stream_, out4, n, 4 * H0, 4 * W0, d.H, d.W, pts, conf); });

        // local features (mpsgraph_engine.mm:425-437): MLP(enc || dec) -> pixel shuffle -> L2 norm
        {
            GemmParams p = gp();
            p.bias = Hh.lf1.b;
            p.act = ACT_GELU;
            p.out = lf1;
            p.ldo = d.lf_hidden;
            launch(kGemm, 2.0 * Tv * Hh.lf1.out * Hh.lf1.in, "lf.fc1", [&] {
                gemm_concat(stream_, d_.dt, 256, EPI_BF16, h0, d.enc_dim, d.enc_dim, h3, d.dec_dim, d.dec_dim, static_cast<int>(Tv),
                            Hh.lf1.w, Hh.lf1.in, Hh.lf1.out, p);
            });
        }
        {
            GemmParams p = gp();
            p.bias = Hh.lf2.b;
            p.out = out_slot(o_desc, d.desc_dim, view, slot);
            p.n_tok = d.ntok;
            p.grid_w = wg;
            p.grid_h = hg;
            p.patch = d.patch;
            const int bn = (d.patch * d.patch) % 8 == 0 ? 192 : 96;
            launch(kGemm, 2.0 * Tv * Hh.lf2.out * Hh.lf2.in, "lf.fc2", [&] {
                gemm_rows(stream_, d_.dt, bn, EPI_DESC, lf1, d.lf_hidden, static_cast<int>(Tv), d.lf_hidden, Hh.lf2.w, d.lf_hidden, Hh.lf2.out, p);
            });
        }
    }

    // The reference's CPU head (mast3r_model.py:86-156), per view: local features =
    // MLP(dec || enc) (the decoder features first, :106-110), of which the first 256
    // channels are the descriptors; pts3d / confidence = conv3x3 + ReLU, conv3x3 + ReLU,
    // conv1x1 of the first 256 decoder channels (:118-131) at patch-grid resolution;
    // both bilinearly upsampled to the image (dpt_head.py:72-116).
    void heads_ref(int view, int n, int slot) {
        const Dims& d = d_;
        const Head& Hh = head[view];
        const long long N = d.ntok, Tv = static_cast<long long>(n) * N;
        const uint16_t* he = enc_out + view * Tv * d.enc_dim;
        const uint16_t* hd = dec_out + view * Tv * d.dec_dim;
        {
            GemmParams p = gp();
            p.bias = Hh.lf1.b;
            p.act = ACT_GELU;
            p.out = lf1;
            p.ldo = d.lf_hidden;
            launch(kGemm, 2.0 * Tv * Hh.lf1.out * Hh.lf1.in, "lf.fc1", [&] {
                gemm_concat(stream_, d_.dt, 256, EPI_BF16, hd, d.dec_dim, d.dec_dim, he, d.enc_dim, d.enc_dim,
                            static_cast<int>(Tv), Hh.lf1.w, Hh.lf1.in, Hh.lf1.out, p);
            });
        }
        linear("lf.fc2", lf1, Tv, Hh.lf2, EPI_F32, rawd, 256);
        // head convs on the first min(256, dec_dim) decoder channels (the tiling of a
        // narrower decoder is folded into the first conv's weights at load time)
        const int c0 = std::min(256, d.dec_dim);
        {
            GemmParams p = gp();
            p.bias = Hh.hd0.b;
            p.act = ACT_RELU;
            p.out = hdg;
            p.ldo = 128;
            const double fl = 2.0 * Tv * 128.0 * 9 * c0;
            launch(kGemm, fl, "head.conv0", [&] {
                gemm_conv3(stream_, d_.dt, 128, EPI_BF16, hd, n, d.hg, d.wg, c0, d.dec_dim, Hh.hd0.w, 128, p);
            });
        }
        conv3("head.conv_out", hdg, n, d.hg, d.wg, 128, Hh.hd2, EPI_HEAD4, out4, ACT_RELU, 128, Hh.w4, Hh.b4);
        float* pts = out_slot(o_pts, 3, view, slot);
        float* conf = out_slot(o_conf, 1, view, slot);
        float* desc = out_slot(o_desc, 256, view, slot);
        launch(kOther, 0, "head.upsample", [&] {
            upsample_ref_split(stream_, out4, n, d.hg, d.wg, d.H, d.W, pts, conf);
            upsample_ref(stream_, rawd, n, d.hg, d.wg, 256, d.H, d.W, desc);
        });
    }

    // Whole inference of n pairs on this device with host buffers: the pairs run in
    // sub-batches of decreasing size (input / output slots first[k] ..), all inputs are copied in first on the
    // copy stream, and each sub-batch's outputs are copied back there as soon as its
    // heads are done, overlapping the next sub-batch's compute.  outs[] point at this
    // device's first pair.  stage_ms[5] (summed over sub-batches), *h2d_ms (input
    // copies), *d2h_ms (output copies, summed) are device times.  Afterwards the input
    // slots hold these n pairs, as after stage().
    // Pageable (not page-locked) caller buffers would make every copy synchronous with
    // the host thread and serialise copies and compute, so they pass through this
    // device's pinned staging slots instead: the inputs in one multi-threaded host copy,
    // the outputs of sub-batch k into slot k % 2, copied on to the caller's arrays by
    // host threads while the GPU computes and copies the next sub-batches.
    static constexpr int kChunkEvents = 8;
    void infer_pipelined(const uint8_t* img1, const uint8_t* img2, int n, float* const outs[6], float* stage_ms,
                         float* h2d_ms, float* d2h_ms) {
        DeviceGuard g(dev_);
        M3R_REQUIRE(n >= 1 && n <= max_pairs_, "infer: pair count out of range for this device");
        // Sub-batches of decreasing size: every sub-batch's output copy overlaps the
        // next one's compute, so only the last copy is exposed -- keep it small; few
        // sub-batches keep the GEMMs and attention at large-batch efficiency (measured at 64
        // pairs: 24/20/16/4 beat 18/18/14/9/5 and 27/21/11/5 end to end).
        static constexpr int kW4[4] = {6, 5, 4, 1}, kW3[3] = {3, 2, 1}, kW2[2] = {2, 1}, kW1[1] = {1};
        const int* w = n >= 40 ? kW4 : n >= 16 ? kW3 : n >= 6 ? kW2 : kW1;
        const int nsub = n >= 40 ? 4 : n >= 16 ? 3 : n >= 6 ? 2 : 1;
        int first[5] = {0}, wsum = 0, wacc = 0;
        for (int k = 0; k < nsub; ++k) wsum += w[k];
        for (int k = 0; k < nsub; ++k) {
            wacc += w[k];
            first[k + 1] = (n * wacc + wsum / 2) / wsum;
        }
        int c = 0;  // largest sub-batch
        for (int k = 0; k < nsub; ++k) c = std::max(c, first[k + 1] - first[k]);
        while (chunk_ev_.size() < static_cast<size_t>(kChunkEvents * nsub + 1)) {
            cudaEvent_t e;
            M3R_CUDA(cudaEventCreate(&e));
            chunk_ev_.push_back(e);
        }
        auto ev = [&](int k, int i) { return chunk_ev_[1 + k * kChunkEvents + i]; };  // i: 0-4 stages, 5 in, 6-7 out
        const size_t ib = static_cast<size_t>(d_.H) * d_.W * 3;
        const size_t px = static_cast<size_t>(d_.H) * d_.W;
        const int per_px[3] = {3, d_.desc_dim, 1};
        const float* bases[3] = {o_pts, o_desc, o_conf};
        const bool in_pageable = is_pageable(img1) || is_pageable(img2);
        bool out_pageable = false;
        for (int i = 0; i < 6; ++i) out_pageable = out_pageable || (outs[i] && is_pageable(outs[i]));
        const size_t pair_out_bytes = sizeof(float) * px * (3 + d_.desc_dim + 1) * 2;
        const bool prof = profiling;
        profiling = false;  // per-launch profiling is a run_resident feature
        try {
            const uint8_t* src1 = img1;
            const uint8_t* src2 = img2;
            if (in_pageable) {
                uint8_t* st = static_cast<uint8_t*>(pinned(stage_in_, stage_in_cap_, 2 * n * ib));
                parallel_memcpy(st, img1, n * ib);
                parallel_memcpy(st + n * ib, img2, n * ib);
                src1 = st;
                src2 = st + n * ib;
            }
            if (out_pageable)
                for (int sslot = 0; sslot < 2; ++sslot) pinned(stage_out_[sslot], stage_out_cap_[sslot], c * pair_out_bytes);
            M3R_CUDA(cudaEventRecord(chunk_ev_[0], copy_stream_));
            for (int k = 0; k < nsub; ++k) {
                const int slot = first[k], nk = first[k + 1] - first[k];
                if (nk <= 0) continue;
                M3R_CUDA(cudaMemcpyAsync(img_slot(0, slot), src1 + slot * ib, nk * ib, cudaMemcpyHostToDevice, copy_stream_));
                M3R_CUDA(cudaMemcpyAsync(img_slot(1, slot), src2 + slot * ib, nk * ib, cudaMemcpyHostToDevice, copy_stream_));
                M3R_CUDA(cudaEventRecord(ev(k, 5), copy_stream_));
            }
            // destination of output kind/view of sub-batch k: the caller's array, or the
            // staging slot k % 2 (laid out as the caller's arrays for nk pairs)
            auto out_dst = [&](int k, int kind, int view, int nk) -> float* {
                const int slot = first[k];
                if (!out_pageable) return outs[2 * kind + view] + slot * px * per_px[kind];
                float* base = static_cast<float*>(stage_out_[k % 2]);
                size_t off = 0;
                for (int q = 0; q < 2 * kind + view; ++q) off += static_cast<size_t>(nk) * px * per_px[q / 2];
                return base + off;
            };
            // staged sub-batch k -> the caller's arrays (host threads)
            auto unstage = [&](int k) {
                const int slot = first[k], nk = first[k + 1] - first[k];
                M3R_CUDA(cudaEventSynchronize(ev(k, 7)));
                for (int kind = 0; kind < 3; ++kind)
                    for (int view = 0; view < 2; ++view)
                        if (outs[2 * kind + view])
                            parallel_memcpy(outs[2 * kind + view] + slot * px * per_px[kind], out_dst(k, kind, view, nk),
                                            sizeof(float) * nk * px * per_px[kind]);
            };
            int last = 0;
            for (int k = 0; k < nsub; ++k) {
                const int slot = first[k], nk = first[k + 1] - first[k];
                if (nk <= 0) continue;
                last = k;
                M3R_CUDA(cudaStreamWaitEvent(stream_, ev(k, 5), 0));
                const cudaEvent_t sev[5] = {ev(k, 0), ev(k, 1), ev(k, 2), ev(k, 3), ev(k, 4)};
                enqueue_forward(nk, slot, sev);
                if (out_pageable && k >= 2) unstage(k - 2);  // frees staging slot k % 2
                M3R_CUDA(cudaStreamWaitEvent(copy_stream_, ev(k, 4), 0));
                M3R_CUDA(cudaEventRecord(ev(k, 6), copy_stream_));
                for (int kind = 0; kind < 3; ++kind)
                    for (int view = 0; view < 2; ++view) {
                        if (!outs[2 * kind + view]) continue;
                        M3R_CUDA(cudaMemcpyAsync(out_dst(k, kind, view, nk), out_slot(bases[kind], per_px[kind], view, slot),
                                                 sizeof(float) * nk * px * per_px[kind], cudaMemcpyDeviceToHost,
                                                 copy_stream_));
                    }
                M3R_CUDA(cudaEventRecord(ev(k, 7), copy_stream_));
            }
            if (out_pageable)
                for (int k = std::max(0, last - 1); k <= last; ++k) unstage(k);
            profiling = prof;
            M3R_CUDA(cudaStreamSynchronize(copy_stream_));
            M3R_CUDA(cudaStreamSynchronize(stream_));
            staged = n;
            check_error();
            for (int i = 0; i < 5; ++i) stage_ms[i] = 0.0f;
            *d2h_ms = 0.0f;
            for (int k = 0; k <= last; ++k) {
                float sm[5];
                const cudaEvent_t sev[5] = {ev(k, 0), ev(k, 1), ev(k, 2), ev(k, 3), ev(k, 4)};
                stage_times(sev, sm);
                for (int i = 0; i < 5; ++i) stage_ms[i] += sm[i];
                float ms;
                M3R_CUDA(cudaEventElapsedTime(&ms, ev(k, 6), ev(k, 7)));
                *d2h_ms += ms;
            }
            M3R_CUDA(cudaEventElapsedTime(h2d_ms, chunk_ev_[0], ev(last, 5)));
        } catch (...) {
            // no copy may still read or write the caller's buffers once the call returns
            profiling = prof;
            cudaStreamSynchronize(copy_stream_);
            cudaStreamSynchronize(stream_);
            cudaGetLastError();
            throw;
        }
    }

    // Retrieval features of k <= 2 * max_pairs images of the model size (encode_retrieval,
    // mpsgraph_engine.mm:1030-1117): the images fill the input slots as view 1 / view 2 of
    // n = ceil(k / 2) pairs (an odd last slot repeats image 0), the patch and encoder stages
    // run over all 2n, then the whitening GEMM (enc_out P + bias, fp32 into the encoder's
    // residual buffer) and the attention weights.  feats [k, N, D], attn [k, N] (host).
    void encode_retrieval(const uint8_t* imgs, int k, float* feats, float* attn) {
        DeviceGuard g(dev_);
        M3R_REQUIRE(k >= 1 && k <= 2 * max_pairs_, "encode_retrieval: image count out of range for this device");
        M3R_REQUIRE(whiten.w != nullptr, "retrieval weights are not loaded (m3r_load_retrieval)");
        const int n = (k + 1) / 2;
        const size_t ib = static_cast<size_t>(d_.H) * d_.W * 3;
        for (int i = 0; i < 2 * n; ++i) {
            const int src = i < k ? i : 0;
            M3R_CUDA(cudaMemcpyAsync(img_slot(i / n, i % n), imgs + src * ib, ib, cudaMemcpyHostToDevice, stream_));
        }
        const bool prof = profiling;
        profiling = false;
        const long long N = d_.ntok, T = 2LL * n * N;
        const int D = d_.enc_dim;
        enqueue_stage(0, n, 0);
        enqueue_stage(1, n, 0);
        linear("ret.whiten", enc_out, T, whiten, EPI_F32, xenc, D);
        retrieval_attention(stream_, xenc, 2 * n, static_cast<int>(N), D, rattn);
        profiling = prof;
        // image i is sequence i of the launch (view 1 slots 0..n-1, then view 2)
        M3R_CUDA(cudaMemcpyAsync(feats, xenc, sizeof(float) * k * N * D, cudaMemcpyDeviceToHost, stream_));
        M3R_CUDA(cudaMemcpyAsync(attn, rattn, sizeof(float) * k * N, cudaMemcpyDeviceToHost, stream_));
        M3R_CUDA(cudaStreamSynchronize(stream_));
        staged = 0;
        check_error();
    }

    // One pair of images of any size: resize + centre crop on the device to the model
    // size (the reference's preprocessing), then the forward pass (slot 0).
    void infer_any(const uint8_t* img1, int h1, int w1, const uint8_t* img2, int h2, int w2, float* const outs[6],
                   float* stage_ms, float* h2d_ms, float* d2h_ms) {
        DeviceGuard g(dev_);
        const size_t b1 = static_cast<size_t>(h1) * w1 * 3, b2 = static_cast<size_t>(h2) * w2 * 3;
        if (raw_cap_ < b1 + b2) {
            if (raw_) M3R_CUDA(cudaFree(raw_));
            raw_ = nullptr;
            raw_cap_ = 0;
            M3R_CUDA(cudaMalloc(&raw_, b1 + b2));
            raw_cap_ = b1 + b2;
        }
        cudaEvent_t* e = stage_ev_;  // 0-4: forward stages, 5-7: copies
        M3R_CUDA(cudaEventRecord(e[5], stream_));
        M3R_CUDA(cudaMemcpyAsync(raw_, img1, b1, cudaMemcpyHostToDevice, stream_));
        M3R_CUDA(cudaMemcpyAsync(raw_ + b1, img2, b2, cudaMemcpyHostToDevice, stream_));
        M3R_CUDA(cudaEventRecord(e[6], stream_));
        resize_crop(stream_, raw_, h1, w1, img_slot(0, 0), d_.H, d_.W);
        resize_crop(stream_, raw_ + b1, h2, w2, img_slot(1, 0), d_.H, d_.W);
        const bool prof = profiling;
        profiling = false;
        float fwd[5];
        try {
            forward(1, fwd);
        } catch (...) {
            profiling = prof;
            throw;
        }
        profiling = prof;
        staged = 1;
        M3R_CUDA(cudaEventElapsedTime(h2d_ms, e[5], e[6]));
        float pre = 0;
        M3R_CUDA(cudaEventElapsedTime(&pre, e[6], stage_ev_[0]));  // resizes (+ queueing)
        for (int i = 0; i < 5; ++i) stage_ms[i] = fwd[i];
        stage_ms[0] += pre;
        const size_t px = static_cast<size_t>(d_.H) * d_.W;
        const int per_px[3] = {3, d_.desc_dim, 1};
        const float* bases[3] = {o_pts, o_desc, o_conf};
        M3R_CUDA(cudaEventRecord(e[6], stream_));
        for (int kind = 0; kind < 3; ++kind)
            for (int view = 0; view < 2; ++view)
                if (outs[2 * kind + view])
                    M3R_CUDA(cudaMemcpyAsync(outs[2 * kind + view], out_slot(bases[kind], per_px[kind], view, 0),
                                             sizeof(float) * px * per_px[kind], cudaMemcpyDeviceToHost, stream_));
        M3R_CUDA(cudaEventRecord(e[7], stream_));
        M3R_CUDA(cudaStreamSynchronize(stream_));
        M3R_CUDA(cudaEventElapsedTime(d2h_ms, e[6], e[7]));
    }

    static bool is_pageable(const void* p) {
        cudaPointerAttributes a;
        if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
            cudaGetLastError();
            return true;
        }
        return a.type == cudaMemoryTypeUnregistered;
    }

    // pinned staging block of at least `need` bytes (kept and grown as needed)
    static void* pinned(void*& p, size_t& cap, size_t need) {
        if (cap < need) {
            if (p) M3R_CUDA(cudaFreeHost(p));
            p = nullptr;
            cap = 0;
            M3R_CUDA(cudaHostAlloc(&p, need, cudaHostAllocPortable));
            cap = need;
        }
        return p;
    }

    void check_error() {
        int e = 0;
        M3R_CUDA(cudaMemcpy(&e, err_, sizeof(int), cudaMemcpyDeviceToHost));
        if (e != 0) {
            M3R_CUDA(cudaMemset(err_, 0, sizeof(int)));
            throw Error(kErrTimeout, "device wait timed out (code " + std::to_string(e) + ")");
        }
    }

    int* err_ptr() const { return err_; }

    // limit of every bounded device wait of this device's launches (0: the default)
    void set_wait_limit(unsigned long long ns) {
        DeviceGuard g(dev_);
        M3R_CUDA(cudaStreamSynchronize(stream_));
        M3R_CUDA(cudaMemcpy(reinterpret_cast<char*>(err_) + offsetof(DevStatus, wait_ns), &ns, sizeof(ns),
                            cudaMemcpyHostToDevice));
    }

private:
    void profiling_reset() { prof_rec_.clear(); }

    int dev_;
    Dims d_;
    int max_pairs_;
    cudaStream_t stream_ = nullptr;
    cudaStream_t copy_stream_ = nullptr;  // host <-> device copies of pipelined infer
    uint8_t* raw_ = nullptr;              // device copies of images of any size (infer_any)
    size_t raw_cap_ = 0;
    void* stage_in_ = nullptr;            // pinned staging of pageable caller buffers
    size_t stage_in_cap_ = 0;
    void* stage_out_[2] = {nullptr, nullptr};
    size_t stage_out_cap_[2] = {0, 0};
    std::vector<cudaEvent_t> chunk_ev_;   // per sub-batch: 5 stage events, input, 2 output-copy events
    int* err_ = nullptr;
    cudaEvent_t stage_ev_[8];
    std::vector<void*> allocs_;
    // forward-stage graphs per (pairs, slot); slot -1 holds the slot-independent stages
    std::map<std::pair<int, int>, std::array<cudaGraphExec_t, 4>> graphs_;
    std::map<std::pair<int, int>, int> direct_runs_;
};

// ---------------------------------------------------------------------------- engine
Engine::Engine(const m3r_config& cfg) : cfg_(cfg), d_(Dims::from(cfg)) {
    M3R_REQUIRE(cfg.max_pairs > 0 && cfg.max_pairs <= 4096, "max_pairs must be in [1, 4096]");
    int ndev = 0;
    M3R_CUDA(cudaGetDeviceCount(&ndev));
    std::vector<int> ids;
    if (cfg.n_devices <= 0) {
        ids.push_back(0);
    } else {
        M3R_REQUIRE(cfg.n_devices <= M3R_MAX_DEVICES, "too many devices");
        for (int i = 0; i < cfg.n_devices; ++i) ids.push_back(cfg.devices[i]);
    }
    for (int id : ids) {
        M3R_REQUIRE(id >= 0 && id < ndev, "device index out of range");
        devs_.emplace_back(new Device(id, d_, cfg.max_pairs));
    }
}

Engine::~Engine() {
    if (!nccl_comms_.empty()) {
        const NcclApi& api = nccl();
        for (void* c : nccl_comms_) api.CommDestroy(static_cast<ncclComm_t>(c));
    }
}

namespace {
// ---------------------------------------------------------------------------- host-side checkpoint
// Every tensor the engine uploads, read from a checkpoint and converted on the host
// (16-bit operand bits, tap-major conv weights, folded norm_y, RoPE tables).
struct HostEnc {
    std::vector<float> n1g, n1b, n2g, n2b;
    HostLin qkv, proj, fc1, fc2;
};
struct HostDec {
    std::vector<float> n[8];
    HostLin qkv, proj, q, kv, cproj, fc1, fc2;
};
struct HostHead {
    HostLin ap0_0, ap0_1t, ap1_0, ap1_1t, ap2_0, ap3_0, ap3_1, rn[4], hd0, hd2, lf1, lf2;
    std::vector<float> w4, b4;
};
struct HostModel {
    HostLin patch;
    std::vector<HostEnc> enc;
    std::vector<float> eng, enb;
    HostLin dembed;
    std::vector<HostDec> dec[2];
    std::vector<float> dng, dnb;
    HostHead hh[2];
    std::vector<float> rope_cos, rope_sin;
};

// Reads and converts a checkpoint for the model `d` (host only; throws Error(kErrIo)
// on a missing, malformed or wrongly-shaped tensor).
HostModel read_model(const std::string& path, const Dims& d) {
    SafetensorsFile f(path);
    const int dt = d.dt;
    HostModel M;
    auto L = [&](const std::string& name, int out, int in, bool bias = true) {
        auto w = f.load_f32(name + ".weight", {out, in});
        std::vector<float> b;
        if (bias) b = f.load_f32(name + ".bias", {out});
        return to16(dt, w, out, in, std::move(b));
    };
    auto V = [&](const std::string& name, int n) { return f.load_f32(name, {n}); };

    // patch embedding [D, 3, p, p] -> [D, kpad]
    const int p = d.patch, kp = 3 * p * p;
    HostLin& patch = M.patch;
    {
        auto w = f.load_f32("patch_embed.proj.weight", {d.enc_dim, 3, p, p});
        std::vector<float> t(static_cast<size_t>(d.enc_dim) * d.kpad, 0.0f);
        for (int o = 0; o < d.enc_dim; ++o)
            for (int kk = 0; kk < kp; ++kk) t[static_cast<size_t>(o) * d.kpad + kk] = w[static_cast<size_t>(o) * kp + kk];
        patch = to16(dt, t, d.enc_dim, d.kpad, V("patch_embed.proj.bias", d.enc_dim));
    }
    std::vector<HostEnc>& enc = M.enc;
    enc.resize(d.enc_depth);
    for (int i = 0; i < d.enc_depth; ++i) {
        const std::string b = "enc_blocks." + std::to_string(i) + ".";
        HostEnc& e = enc[i];
        e.n1g = V(b + "norm1.weight", d.enc_dim);
        e.n1b = V(b + "norm1.bias", d.enc_dim);
        e.n2g = V(b + "norm2.weight", d.enc_dim);
        e.n2b = V(b + "norm2.bias", d.enc_dim);
        e.qkv = L(b + "attn.qkv", 3 * d.enc_dim, d.enc_dim);
        e.proj = L(b + "attn.proj", d.enc_dim, d.enc_dim);
        e.fc1 = L(b + "mlp.fc1", d.enc_mlp, d.enc_dim);
        e.fc2 = L(b + "mlp.fc2", d.enc_dim, d.enc_mlp);
    }
    M.eng = V("enc_norm.weight", d.enc_dim);
    M.enb = V("enc_norm.bias", d.enc_dim);
    M.dembed = L("decoder_embed", d.dec_dim, d.enc_dim);
    std::vector<HostDec>* dec = M.dec;
    const int Dd = d.dec_dim;
    for (int view = 0; view < 2; ++view) {
        dec[view].resize(d.dec_depth);
        for (int i = 0; i < d.dec_depth; ++i) {
            const std::string b = (view == 0 ? "dec_blocks." : "dec_blocks2.") + std::to_string(i) + ".";
            HostDec& e = dec[view][i];
            const char* norms[4] = {"norm1", "norm2", "norm_y", "norm3"};
            for (int k = 0; k < 4; ++k) {
                e.n[2 * k] = V(b + norms[k] + ".weight", Dd);
                e.n[2 * k + 1] = V(b + norms[k] + ".bias", Dd);
            }
            e.qkv = L(b + "attn.qkv", 3 * Dd, Dd);
            e.proj = L(b + "attn.proj", Dd, Dd);
            e.q = L(b + "cross_attn.projq", Dd, Dd);
            {
                auto wk = f.load_f32(b + "cross_attn.projk.weight", {Dd, Dd});
                auto wv = f.load_f32(b + "cross_attn.projv.weight", {Dd, Dd});
                auto bk = V(b + "cross_attn.projk.bias", Dd);
                auto bv = V(b + "cross_attn.projv.bias", Dd);
                wk.insert(wk.end(), wv.begin(), wv.end());
                bk.insert(bk.end(), bv.begin(), bv.end());
                // norm_y's affine part folded into the K/V projection:
                //   (yhat * g + beta) W^T + b = yhat (W diag(g))^T + (b + W beta),
                // so the normalisation yhat of the other view's projected encoder output
                // (the same input for every block) is computed once per pass
                const std::vector<float>& gy = e.n[4];
                const std::vector<float>& by = e.n[5];
                for (int o = 0; o < 2 * Dd; ++o) {
                    double acc = bk[o];
                    for (int i = 0; i < Dd; ++i) acc += static_cast<double>(wk[static_cast<size_t>(o) * Dd + i]) * by[i];
                    bk[o] = static_cast<float>(acc);
                    for (int i = 0; i < Dd; ++i) wk[static_cast<size_t>(o) * Dd + i] *= gy[i];
                }
                e.kv = to16(dt, wk, 2 * Dd, Dd, bk);
            }
            e.cproj = L(b + "cross_attn.proj", Dd, Dd);
            e.fc1 = L(b + "mlp.fc1", d.dec_mlp, Dd);
            e.fc2 = L(b + "mlp.fc2", Dd, d.dec_mlp);
        }
    }
    M.dng = V("dec_norm.weight", Dd);
    M.dnb = V("dec_norm.bias", Dd);
    HostHead* hh = M.hh;
    const int dpt[4] = {96, 192, 384, 768};
    for (int view = 0; view < 2; ++view) {
        const std::string t = std::string(view == 0 ? "downstream_head1" : "downstream_head2") + ".dpt.";
        HostHead& H = hh[view];
        const std::string lf = std::string(view == 0 ? "downstream_head1" : "downstream_head2") + ".head_local_features.";
        if (d.head == M3R_HEAD_REF_SIMPLE) {
            // mast3r_model.py:86-156: head.0 / head.2 / head.4 on the first 256 decoder
            // channels (a decoder narrower than 256 is tiled, :120-125: its tiling is folded
            // into head.0's weights); descriptors = the first 256 outputs of the local
            // features' fc2 (:139-146), whose fc1 reads (decoder || encoder) (:106-110)
            const int c0 = std::min(256, Dd);
            auto w0 = f.load_f32(t + "head.0.weight", {128, 256, 3, 3});
            std::vector<float> folded(static_cast<size_t>(128) * c0 * 9, 0.0f);
            for (int o = 0; o < 128; ++o)
                for (int k = 0; k < 256; ++k)
                    for (int tap = 0; tap < 9; ++tap)
                        folded[(static_cast<size_t>(o) * c0 + k % Dd) * 9 + tap] += w0[(static_cast<size_t>(o) * 256 + k) * 9 + tap];
            H.hd0 = conv3_weights(dt, folded, 128, c0, V(t + "head.0.bias", 128));
            H.hd2 = conv3_weights(dt, f.load_f32(t + "head.2.weight", {128, 128, 3, 3}), 128, 128, V(t + "head.2.bias", 128));
            H.w4 = f.load_f32(t + "head.4.weight", {4, 128, 1, 1});
            H.b4 = V(t + "head.4.bias", 4);
            H.lf1 = L(lf + "fc1", d.lf_hidden, Dd + d.enc_dim);
            const int rows = 25 * p * p;  // the checkpoint's fc2: (24 + 1) p^2 outputs
            M3R_REQUIRE(rows >= 256, "local-feature head has fewer than 256 outputs");
            auto w = f.load_f32(lf + "fc2.weight", {rows, d.lf_hidden});
            auto b = V(lf + "fc2.bias", rows);
            w.resize(static_cast<size_t>(256) * d.lf_hidden);
            b.resize(256);
            H.lf2 = to16(dt, w, 256, d.lf_hidden, b);
            continue;
        }
        auto conv1 = [&](const std::string& name, int out, int in) {
            auto w = f.load_f32(name + ".weight", {out, in, 1, 1});
            return to16(dt, w, out, in, V(name + ".bias", out));
        };
        H.ap0_0 = conv1(t + "act_postprocess.0.0", 96, d.enc_dim);
        H.ap0_1t = convt_weights(dt, f.load_f32(t + "act_postprocess.0.1.weight", {96, 96, 4, 4}), 96, 96, 4,
                                 V(t + "act_postprocess.0.1.bias", 96));
        H.ap1_0 = conv1(t + "act_postprocess.1.0", 192, Dd);
        H.ap1_1t = convt_weights(dt, f.load_f32(t + "act_postprocess.1.1.weight", {192, 192, 2, 2}), 192, 192, 2,
                                 V(t + "act_postprocess.1.1.bias", 192));
        H.ap2_0 = conv1(t + "act_postprocess.2.0", 384, Dd);
        H.ap3_0 = conv1(t + "act_postprocess.3.0", 768, Dd);
        H.ap3_1 = conv3_weights(dt, f.load_f32(t + "act_postprocess.3.1.weight", {768, 768, 3, 3}), 768, 768,
                                V(t + "act_postprocess.3.1.bias", 768));
        for (int k = 0; k < 4; ++k)
            H.rn[k] = conv3_weights(dt, f.load_f32(t + "scratch.layer_rn." + std::to_string(k) + ".weight", {256, dpt[k], 3, 3}),
                                    256, dpt[k]);
        H.hd0 = conv3_weights(dt, f.load_f32(t + "head.0.weight", {128, 256, 3, 3}), 128, 256, V(t + "head.0.bias", 128));
        H.hd2 = conv3_weights(dt, f.load_f32(t + "head.2.weight", {128, 128, 3, 3}), 128, 128, V(t + "head.2.bias", 128));
        H.w4 = f.load_f32(t + "head.4.weight", {4, 128, 1, 1});
        H.b4 = V(t + "head.4.bias", 4);
        H.lf1 = L(lf + "fc1", d.lf_hidden, d.enc_dim + Dd);
        {
            // keep the desc_dim descriptor channels of every (dy, dx) group of desc_dim + 1
            // (the extra channel is the discarded descriptor confidence)
            const int groups = p * p, cin = d.desc_dim + 1;
            auto w = f.load_f32(lf + "fc2.weight", {groups * cin, d.lf_hidden});
            auto b = V(lf + "fc2.bias", groups * cin);
            std::vector<float> w2(static_cast<size_t>(groups) * d.desc_dim * d.lf_hidden), b2(static_cast<size_t>(groups) * d.desc_dim);
            for (int g = 0; g < groups; ++g)
                for (int c = 0; c < d.desc_dim; ++c) {
                    const size_t src = static_cast<size_t>(g) * cin + c, dst = static_cast<size_t>(g) * d.desc_dim + c;
                    std::memcpy(&w2[dst * d.lf_hidden], &w[src * d.lf_hidden], sizeof(float) * d.lf_hidden);
                    b2[dst] = b[src];
                }
            H.lf2 = to16(dt, w2, groups * d.desc_dim, d.lf_hidden, b2);
        }
    }
    // RoPE tables (rope2d.py:77-92): freq_i = 1 / 100^(i/16), angle = pos * freq_i in float32;
    // frequency-major [16][maxpos] (the QKV epilogue reads a warp's consecutive tokens)
    const int maxpos = std::max(d.hg, d.wg);
    std::vector<float>& rc = M.rope_cos;
    std::vector<float>& rs = M.rope_sin;
    rc.assign(static_cast<size_t>(maxpos) * 16, 0.0f);
    rs.assign(static_cast<size_t>(maxpos) * 16, 0.0f);
    for (int i = 0; i < 16; ++i) {
        const float freq = 1.0f / std::pow(100.0f, static_cast<float>(i) / 16.0f);
        for (int pos = 0; pos < maxpos; ++pos) {
            const float ang = static_cast<float>(pos) * freq;
            rc[static_cast<size_t>(i) * maxpos + pos] = static_cast<float>(std::cos(static_cast<double>(ang)));
            rs[static_cast<size_t>(i) * maxpos + pos] = static_cast<float>(std::sin(static_cast<double>(ang)));
        }
    }

    return M;
}
}  // namespace

void check_checkpoint(const std::string& path, const Dims& d) { (void)read_model(path, d); }

void Engine::load(const std::string& path) {
    const HostModel M = read_model(path, d_);
    const Dims& d = d_;
    const int Dd = d.dec_dim;
    const HostLin& patch = M.patch;
    const std::vector<HostEnc>& enc = M.enc;
    const std::vector<float>&eng = M.eng, &enb = M.enb, &dng = M.dng, &dnb = M.dnb;
    const HostLin& dembed = M.dembed;
    const std::vector<HostDec>* dec = M.dec;
    const HostHead* hh = M.hh;
    const std::vector<float>&rc = M.rope_cos, &rs = M.rope_sin;
    // upload to every device
    for (auto& dp : devs_) {
        Device& D = *dp;
        DeviceGuard g(D.dev());
        D.patch = D.upload(patch);
        D.enc.resize(d.enc_depth);
        for (int i = 0; i < d.enc_depth; ++i) {
            EncBlock& B = D.enc[i];
            B.n1 = D.upload_norm(enc[i].n1g, enc[i].n1b);
            B.n2 = D.upload_norm(enc[i].n2g, enc[i].n2b);
            B.qkv = D.upload(enc[i].qkv);
            B.proj = D.upload(enc[i].proj);
            B.fc1 = D.upload(enc[i].fc1);
            B.fc2 = D.upload(enc[i].fc2);
        }
        D.enc_norm = D.upload_norm(eng, enb);
        D.dec_embed = D.upload(dembed);
        for (int view = 0; view < 2; ++view) {
            D.dec[view].resize(d.dec_depth);
            for (int i = 0; i < d.dec_depth; ++i) {
                const HostDec& e = dec[view][i];
                DecBlock& B = D.dec[view][i];
                B.n1 = D.upload_norm(e.n[0], e.n[1]);
                B.n2 = D.upload_norm(e.n[2], e.n[3]);
                B.n3 = D.upload_norm(e.n[6], e.n[7]);
                B.qkv = D.upload(e.qkv);
                B.proj = D.upload(e.proj);
                B.q = D.upload(e.q);
                B.kv = D.upload(e.kv);
                B.cproj = D.upload(e.cproj);
                B.fc1 = D.upload(e.fc1);
                B.fc2 = D.upload(e.fc2);
            }
        }
        D.dec_norm = D.upload_norm(dng, dnb);
        D.unit_norm = D.upload_norm(std::vector<float>(Dd, 1.0f), std::vector<float>(Dd, 0.0f));
        for (int view = 0; view < 2; ++view) {
            const HostHead& H = hh[view];
            Head& O = D.head[view];
            O.ap0_0 = D.upload(H.ap0_0);
            O.ap0_1t = D.upload(H.ap0_1t);
            O.ap1_0 = D.upload(H.ap1_0);
            O.ap1_1t = D.upload(H.ap1_1t);
            O.ap2_0 = D.upload(H.ap2_0);
            O.ap3_0 = D.upload(H.ap3_0);
            O.ap3_1 = D.upload(H.ap3_1);
            for (int k = 0; k < 4; ++k) O.rn[k] = D.upload(H.rn[k]);
            O.hd0 = D.upload(H.hd0);
            O.hd2 = D.upload(H.hd2);
            O.w4 = D.upload(H.w4);
            O.b4 = D.upload(H.b4);
            O.lf1 = D.upload(H.lf1);
            O.lf2 = D.upload(H.lf2);
        }
        D.rope_cos = D.upload(rc);
        D.rope_sin = D.upload(rs);
        M3R_CUDA(cudaDeviceSynchronize());
    }
    ready_ = true;
}

std::vector<std::pair<int, int>> Engine::shards(int n_pairs) const {
    std::vector<std::pair<int, int>> s;
    const int nd = static_cast<int>(devs_.size());
    int first = 0;
    for (int i = 0; i < nd; ++i) {
        const int cnt = n_pairs / nd + (i < n_pairs % nd ? 1 : 0);
        s.push_back({first, cnt});
        first += cnt;
    }
    return s;
}

namespace {
// Runs fn(i) for every device on its own host thread; rethrows the first error.
void for_each_device(size_t n, const std::function<void(size_t)>& fn) {
    if (n == 1) {
        fn(0);
        return;
    }
    std::vector<std::thread> th;
    std::vector<std::exception_ptr> errs(n);
    for (size_t i = 0; i < n; ++i)
        th.emplace_back([&, i] {
            try {
                fn(i);
            } catch (...) {
                errs[i] = std::current_exception();
            }
        });
    for (auto& t : th) t.join();
    for (auto& e : errs)
        if (e) std::rethrow_exception(e);
}
}  // namespace

void Engine::stage(const uint8_t* img1, const uint8_t* img2, int n_pairs) {
    if (!ready_) throw Error(kErrState, "engine is not loaded");
    M3R_REQUIRE(n_pairs >= 1, "n_pairs must be >= 1");
    const auto sh = shards(n_pairs);
    const size_t img_bytes = static_cast<size_t>(d_.H) * d_.W * 3;
    for (size_t i = 0; i < devs_.size(); ++i)
        M3R_REQUIRE(sh[i].second <= cfg_.max_pairs, "too many pairs for one device launch (raise max_pairs)");
    for_each_device(devs_.size(), [&](size_t i) {
        Device& D = *devs_[i];
        DeviceGuard g(D.dev());
        const int first = sh[i].first, cnt = sh[i].second;
        D.staged = cnt;
        if (cnt == 0) return;
        M3R_CUDA(cudaMemcpyAsync(D.img_slot(0, 0), img1 + first * img_bytes, cnt * img_bytes, cudaMemcpyHostToDevice,
                                 D.stream()));
        M3R_CUDA(cudaMemcpyAsync(D.img_slot(1, 0), img2 + first * img_bytes, cnt * img_bytes, cudaMemcpyHostToDevice,
                                 D.stream()));
        M3R_CUDA(cudaStreamSynchronize(D.stream()));
    });
    staged_pairs_ = n_pairs;
}

float Engine::run_resident(int n_pairs, float* stage_ms) {
    if (!ready_) throw Error(kErrState, "engine is not loaded");
    if (n_pairs != staged_pairs_) throw Error(kErrState, "run_resident: pair count differs from the staged inputs");
    std::vector<float> ms(devs_.size() * 5, 0.0f);
    for_each_device(devs_.size(), [&](size_t i) {
        Device& D = *devs_[i];
        D.profiling = profiling_ && i == 0;
        if (D.staged > 0) D.forward(D.staged, &ms[i * 5]);
    });
    float mx = 0.0f;
    for (size_t i = 0; i < devs_.size(); ++i) {
        mx = std::max(mx, ms[i * 5 + 4]);
        if (stage_ms && (i == 0 || ms[i * 5 + 4] >= mx))
            for (int k = 0; k < 5; ++k) stage_ms[k] = ms[i * 5 + k];
    }
    return mx;
}

void Engine::fetch(int n_pairs, float* const outs[6]) {
    if (n_pairs != staged_pairs_) throw Error(kErrState, "fetch: pair count differs from the staged inputs");
    const auto sh = shards(n_pairs);
    const size_t px = static_cast<size_t>(d_.H) * d_.W;
    for_each_device(devs_.size(), [&](size_t i) {
        Device& D = *devs_[i];
        DeviceGuard g(D.dev());
        const int first = sh[i].first, cnt = sh[i].second;
        if (cnt == 0) return;
        const int per_px[3] = {3, d_.desc_dim, 1};
        const float* src[3] = {D.o_pts, D.o_desc, D.o_conf};
        for (int k = 0; k < 3; ++k)
            for (int view = 0; view < 2; ++view) {
                float* dst = outs[2 * k + view];
                if (!dst) continue;
                M3R_CUDA(cudaMemcpyAsync(dst + first * px * per_px[k], D.out_slot(src[k], per_px[k], view, 0),
                                         sizeof(float) * cnt * px * per_px[k], cudaMemcpyDeviceToHost, D.stream()));
            }
        M3R_CUDA(cudaStreamSynchronize(D.stream()));
    });
}

void Engine::infer(const uint8_t* img1, const uint8_t* img2, int n_pairs, float* const outs[6], float* timing) {
    if (!ready_) throw Error(kErrState, "engine is not loaded");
    M3R_REQUIRE(n_pairs >= 1, "n_pairs must be >= 1");
    const auto t0 = std::chrono::steady_clock::now();
    float st[5] = {0, 0, 0, 0, 0};
    float h2d = 0, d2h = 0;
    std::mutex mu;
    const size_t ib = static_cast<size_t>(d_.H) * d_.W * 3;
    const size_t px = static_cast<size_t>(d_.H) * d_.W;
    const int per_px[3] = {3, d_.desc_dim, 1};
    // launches of up to max_pairs per device; every device pipelines its share
    // (sub-batches whose output copies overlap the next sub-batch's compute)
    const int per_launch = cfg_.max_pairs * static_cast<int>(devs_.size());
    for (int first = 0; first < n_pairs; first += per_launch) {
        const int cnt = std::min(per_launch, n_pairs - first);
        const auto sh = shards(cnt);
        float launch_st[5] = {0, 0, 0, 0, 0}, launch_h2d = 0, launch_d2h = 0;
        for_each_device(devs_.size(), [&](size_t i) {
            const int f = first + sh[i].first, c = sh[i].second;
            devs_[i]->staged = c;
            if (c == 0) return;
            float* o[6];
            for (int k = 0; k < 3; ++k)
                for (int view = 0; view < 2; ++view)
                    o[2 * k + view] = outs[2 * k + view] ? outs[2 * k + view] + f * px * per_px[k] : nullptr;
            float sm[5], hm = 0, dm = 0;
            devs_[i]->infer_pipelined(img1 + f * ib, img2 + f * ib, c, o, sm, &hm, &dm);
            std::lock_guard<std::mutex> lk(mu);  // the slowest device sets the launch's times
            if (sm[4] >= launch_st[4])
                for (int k = 0; k < 5; ++k) launch_st[k] = sm[k];
            launch_h2d = std::max(launch_h2d, hm);
            launch_d2h = std::max(launch_d2h, dm);
        });
        for (int k = 0; k < 5; ++k) st[k] += launch_st[k];
        h2d += launch_h2d;
        d2h += launch_d2h;
        staged_pairs_ = cnt;  // the input slots hold this launch's pairs, as after stage()
    }
    if (timing) {
        timing[M3R_T_PREPROCESS] = st[0];
        timing[M3R_T_ENCODER] = st[1];
        timing[M3R_T_DECODER] = st[2];
        timing[M3R_T_HEADS] = st[3];
        timing[M3R_T_H2D] = h2d;
        timing[M3R_T_D2H] = d2h;
        timing[M3R_T_INFERENCE] = st[4];
        timing[M3R_T_TOTAL] =
            static_cast<float>(std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count());
    }
}

void Engine::load_retrieval(const std::string& path) {
    if (!ready_) throw Error(kErrState, "load the model before the retrieval weights");
    SafetensorsFile f(path);
    const int D = d_.enc_dim;
    const std::vector<float> m = f.load_f32("prewhiten.m", {D});
    const std::vector<float> P = f.load_f32("prewhiten.p", {D, D});
    // (x - m) P = x P - m P: the GEMM's weight is P^T ([out, in]) and its bias -(m P)
    std::vector<float> wt(static_cast<size_t>(D) * D), bias(D);
    for (int j = 0; j < D; ++j) {
        double acc = 0.0;
        for (int i = 0; i < D; ++i) {
            wt[static_cast<size_t>(j) * D + i] = P[static_cast<size_t>(i) * D + j];
            acc += static_cast<double>(m[i]) * P[static_cast<size_t>(i) * D + j];
        }
        bias[j] = static_cast<float>(-acc);
    }
    const HostLin h = to16(d_.dt, wt, D, D, bias);
    for (auto& dp : devs_) {
        DeviceGuard g(dp->dev());
        dp->whiten = dp->upload(h);
        M3R_CUDA(cudaDeviceSynchronize());
    }
    retrieval_ready_ = true;
}

void Engine::encode_retrieval(const uint8_t* imgs, int k, float* feats, float* attn, float* timing) {
    if (!ready_ || !retrieval_ready_) throw Error(kErrState, "retrieval weights are not loaded");
    M3R_REQUIRE(imgs && feats && attn && k >= 1, "encode_retrieval: bad arguments");
    const auto t0 = std::chrono::steady_clock::now();
    const size_t ib = static_cast<size_t>(d_.H) * d_.W * 3;
    const size_t fb = static_cast<size_t>(d_.ntok) * d_.enc_dim;
    const int per = 2 * cfg_.max_pairs;
    for (int first = 0; first < k; first += per) {
        const int c = std::min(per, k - first);
        devs_[0]->encode_retrieval(imgs + first * ib, c, feats + first * fb, attn + static_cast<size_t>(first) * d_.ntok);
    }
    staged_pairs_ = 0;
    if (timing) {
        for (int i = 0; i < M3R_T_COUNT; ++i) timing[i] = 0.0f;
        timing[M3R_T_TOTAL] =
            static_cast<float>(std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count());
    }
}

void Engine::infer_any(const uint8_t* img1, int h1, int w1, const uint8_t* img2, int h2, int w2, float* const outs[6],
                       float* timing) {
    if (!ready_) throw Error(kErrState, "engine is not loaded");
    M3R_REQUIRE(img1 && img2 && h1 > 0 && w1 > 0 && h2 > 0 && w2 > 0, "infer_any: bad image");
    const auto t0 = std::chrono::steady_clock::now();
    float st[5] = {0, 0, 0, 0, 0}, h2d = 0, d2h = 0;
    devs_[0]->infer_any(img1, h1, w1, img2, h2, w2, outs, st, &h2d, &d2h);
    for (size_t i = 1; i < devs_.size(); ++i) devs_[i]->staged = 0;
    staged_pairs_ = 1;
    if (timing) {
        timing[M3R_T_PREPROCESS] = st[0];
        timing[M3R_T_ENCODER] = st[1];
        timing[M3R_T_DECODER] = st[2];
        timing[M3R_T_HEADS] = st[3];
        timing[M3R_T_H2D] = h2d;
        timing[M3R_T_D2H] = d2h;
        timing[M3R_T_INFERENCE] = st[4];
        timing[M3R_T_TOTAL] =
            static_cast<float>(std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count());
    }
}

std::string Engine::profile_ops() const {
    std::string t;
    char line[256];
    for (const auto& o : devs_[0]->prof_ops) {
        std::snprintf(line, sizeof(line), "%s\t%.6f\t%.6e\t%ld\n", o.op.c_str(), o.ms, o.flops, o.launches);
        t += line;
    }
    return t;
}

void Engine::set_wait_timeout(unsigned long long ns) {
    for (auto& d : devs_) d->set_wait_limit(ns);
}

void Engine::profile(double* out) const {
    const Device& D = *devs_[0];
    out[0] = D.prof.ms[0];
    out[1] = D.prof.flops[0];
    out[2] = D.prof.ms[1];
    out[3] = D.prof.flops[1];
    out[4] = D.prof.ms[2];
    out[5] = static_cast<double>(D.prof.launches[0]);
    out[6] = static_cast<double>(D.prof.launches[1]);
    out[7] = static_cast<double>(D.prof.launches[2]);
}

// ---------------------------------------------------------------------------- match
namespace {
// Four events around the device phases of one match: normalize, arg-max, select.
struct MatchEvents {
    cudaEvent_t e[4] = {nullptr, nullptr, nullptr, nullptr};
    MatchEvents() {
        for (auto& x : e) M3R_CUDA(cudaEventCreate(&x));
    }
    ~MatchEvents() {
        for (auto& x : e)
            if (x) cudaEventDestroy(x);
    }
    MatchEvents(const MatchEvents&) = delete;
    MatchEvents& operator=(const MatchEvents&) = delete;
    // ms[0..2] per phase, ms[3] all three (the events must have completed)
    void phases(float* ms) const {
        for (int i = 0; i < 3; ++i) M3R_CUDA(cudaEventElapsedTime(&ms[i], e[i], e[i + 1]));
        M3R_CUDA(cudaEventElapsedTime(&ms[3], e[0], e[3]));
    }
};
}  // namespace

int Engine::match(const float* d1, const float* d2, int hh, int ww, int dd, int top_k, int reciprocal, float thr,
                  int64_t* idx1, int64_t* idx2, float* conf, float* p1, float* p2, float* timing,
                  const MatchExtras* ex) {
    const bool weighted = ex && ex->conf_1 && ex->conf_2;
    const auto t0 = std::chrono::steady_clock::now();
    M3R_REQUIRE(hh >= 0 && ww >= 0 && dd > 0 && top_k >= 0, "match: bad arguments");
    const long long n = static_cast<long long>(hh) * ww;
    M3R_REQUIRE(n < 0x7FFFFFFFLL, "match: too many descriptors");
    if (n == 0 || top_k == 0) {
        if (timing) timing[M3R_T_TOTAL] = 0.0f;
        return 0;
    }
    int m = 0;
    float phase_ms[4] = {0, 0, 0, 0};  // normalize, arg-max, select, all three (device time)
    if (devs_.size() > 1 && n >= static_cast<long long>(devs_.size()) * 128) {
        m = match_multi(d1, d2, weighted ? ex->conf_1 : nullptr, weighted ? ex->conf_2 : nullptr, n, ww, dd, top_k,
                        reciprocal, thr, idx1, idx2, conf, phase_ms);
    } else {
        // single device (device 0 of the engine)
        Device& D = *devs_[0];
        DeviceGuard g(D.dev());
        cudaStream_t s = D.stream();
        D.mws.reserve(n, dd);
        MatchEvents ev;
        M3R_CUDA(cudaMemcpyAsync(D.mws.a, d1, sizeof(float) * n * dd, cudaMemcpyHostToDevice, s));
        M3R_CUDA(cudaMemcpyAsync(D.mws.b, d2, sizeof(float) * n * dd, cudaMemcpyHostToDevice, s));
        if (weighted) {
            M3R_CUDA(cudaMemcpyAsync(D.mws.c1, ex->conf_1, sizeof(float) * n, cudaMemcpyHostToDevice, s));
            M3R_CUDA(cudaMemcpyAsync(D.mws.c2, ex->conf_2, sizeof(float) * n, cudaMemcpyHostToDevice, s));
        }
        M3R_CUDA(cudaEventRecord(ev.e[0], s));
        match_normalize2(s, D.mws.a, D.mws.a, n, D.mws.b, D.mws.b, n, dd);
        M3R_CUDA(cudaEventRecord(ev.e[1], s));
        match_argmax(s, D.mws.a, D.mws.b, 0, n, n, dd, D.mws.rowkey, D.mws.colkey, true,
                     weighted ? D.mws.c1 : nullptr, weighted ? D.mws.c2 : nullptr);
        M3R_CUDA(cudaEventRecord(ev.e[2], s));
        m = match_select(s, D.mws, n, 0, reciprocal, thr, top_k);
        M3R_CUDA(cudaEventRecord(ev.e[3], s));
        if (m > 0) {
            M3R_CUDA(cudaMemcpyAsync(idx1, D.mws.idx1, sizeof(int64_t) * m, cudaMemcpyDeviceToHost, s));
            M3R_CUDA(cudaMemcpyAsync(idx2, D.mws.idx2, sizeof(int64_t) * m, cudaMemcpyDeviceToHost, s));
            M3R_CUDA(cudaMemcpyAsync(conf, D.mws.conf, sizeof(float) * m, cudaMemcpyDeviceToHost, s));
        }
        M3R_CUDA(cudaStreamSynchronize(s));
        ev.phases(phase_ms);
    }
    for (int i = 0; i < m; ++i) {  // matching.cpp:216-222
        p1[2 * i] = static_cast<float>(idx1[i] % ww);
        p1[2 * i + 1] = static_cast<float>(idx1[i] / ww);
        p2[2 * i] = static_cast<float>(idx2[i] % ww);
        p2[2 * i + 1] = static_cast<float>(idx2[i] / ww);
    }
    // 3-D points of the matches (matching.py:144-152; zeros without pts3d maps, as the
    // C++ path returns, matching.cpp:231-232)
    if (ex && ex->out3_1 && ex->out3_2) {
        const bool have = ex->pts3d_1 && ex->pts3d_2;
        for (int i = 0; i < m; ++i)
            for (int q = 0; q < 3; ++q) {
                ex->out3_1[3 * i + q] = have ? ex->pts3d_1[3 * idx1[i] + q] : 0.0f;
                ex->out3_2[3 * i + q] = have ? ex->pts3d_2[3 * idx2[i] + q] : 0.0f;
            }
    }
    if (timing) {
        for (int i = 0; i < M3R_T_COUNT; ++i) timing[i] = 0.0f;
        timing[M3R_T_MATCH_NORMALIZE] = phase_ms[0];
        timing[M3R_T_MATCH_ARGMAX] = phase_ms[1];
        timing[M3R_T_MATCH_SELECT] = phase_ms[2];
        timing[M3R_T_INFERENCE] = phase_ms[3];
        timing[M3R_T_TOTAL] =
            static_cast<float>(std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count());
    }
    return m;
}

// Rows of A sharded over the devices; B replicated.  Each device finds exact row
// maxima for its rows and column maxima over its rows; the column keys (max value,
// lowest row) are max-reduced over the devices with NCCL (in place, over NVLink), so
// every device then holds the exact nn_21 and runs the reciprocal test, threshold and
// top-k on its own rows.  The per-device results (each <= top_k, exact top-k of its
// rows) are merged on the host: the global top-k is inside their union.
int Engine::match_multi(const float* d1, const float* d2, const float* c1, const float* c2, long long n, int ww, int dd,
                        int top_k, int reciprocal, float thr, int64_t* idx1, int64_t* idx2, float* conf,
                        float* phase_ms) {
    const int nd = static_cast<int>(devs_.size());
    const NcclApi& api = nccl();
    if (nccl_comms_.empty()) {
        std::vector<ncclComm_t> comms(nd);
        std::vector<int> ids(nd);
        for (int i = 0; i < nd; ++i) ids[i] = devs_[i]->dev();
        nccl_check(api.CommInitAll(comms.data(), nd, ids.data()), "ncclCommInitAll");
        for (auto c : comms) nccl_comms_.push_back(c);
    }
    struct Part {
        long long r0 = 0, r1 = 0;
        int m = 0, total = 0;
        std::vector<int64_t> i1, i2;
        std::vector<float> c;
        std::unique_ptr<MatchEvents> ev;  // created with the part's device current
    };
    std::vector<Part> parts(nd);
    for (int i = 0; i < nd; ++i) {
        parts[i].r0 = n * i / nd;
        parts[i].r1 = n * (i + 1) / nd;
    }
    // phase 1: copy in, normalise, arg-max over the device's rows
    for_each_device(devs_.size(), [&](size_t i) {
        Device& D = *devs_[i];
        Part& P = parts[i];
        DeviceGuard g(D.dev());
        cudaStream_t s = D.stream();
        const long long nr = P.r1 - P.r0;
        D.mws.reserve(n, dd);
        P.ev.reset(new MatchEvents());
        M3R_CUDA(cudaMemcpyAsync(D.mws.a, d1 + P.r0 * dd, sizeof(float) * nr * dd, cudaMemcpyHostToDevice, s));
        M3R_CUDA(cudaMemcpyAsync(D.mws.b, d2, sizeof(float) * n * dd, cudaMemcpyHostToDevice, s));
        if (c1 && c2) {  // whole maps: conf_1 is addressed by global row
            M3R_CUDA(cudaMemcpyAsync(D.mws.c1, c1, sizeof(float) * n, cudaMemcpyHostToDevice, s));
            M3R_CUDA(cudaMemcpyAsync(D.mws.c2, c2, sizeof(float) * n, cudaMemcpyHostToDevice, s));
        }
        M3R_CUDA(cudaEventRecord(P.ev->e[0], s));
        match_normalize2(s, D.mws.a, D.mws.a, nr, D.mws.b, D.mws.b, n, dd);
        M3R_CUDA(cudaEventRecord(P.ev->e[1], s));
        // A is addressed by global row: rows [r0, r1) live at mws.a[0 .. nr)
        match_argmax(s, D.mws.a - P.r0 * dd, D.mws.b, P.r0, P.r1, n, dd, D.mws.rowkey, D.mws.colkey, true,
                     c1 && c2 ? D.mws.c1 : nullptr, c1 && c2 ? D.mws.c2 : nullptr);
        M3R_CUDA(cudaEventRecord(P.ev->e[2], s));
    });
    // phase 2: column keys max-reduced over the devices
    nccl_check(api.GroupStart(), "ncclGroupStart");
    for (int i = 0; i < nd; ++i) {
        Device& D = *devs_[i];
        DeviceGuard g(D.dev());
        nccl_check(api.AllReduce(D.mws.colkey, D.mws.colkey, static_cast<size_t>(n), ncclUint64, ncclMax,
                                 static_cast<ncclComm_t>(nccl_comms_[i]), D.stream()),
                   "ncclAllReduce(column keys)");
    }
    nccl_check(api.GroupEnd(), "ncclGroupEnd");
    // phase 3: reciprocal test, threshold and top-k per shard, results to the host
    for_each_device(devs_.size(), [&](size_t i) {
        Device& D = *devs_[i];
        Part& P = parts[i];
        DeviceGuard g(D.dev());
        cudaStream_t s = D.stream();
        P.m = match_select(s, D.mws, P.r1 - P.r0, P.r0, reciprocal, thr, top_k, &P.total);
        M3R_CUDA(cudaEventRecord(P.ev->e[3], s));
        P.i1.resize(P.m);
        P.i2.resize(P.m);
        P.c.resize(P.m);
        if (P.m > 0) {
            M3R_CUDA(cudaMemcpyAsync(P.i1.data(), D.mws.idx1, sizeof(int64_t) * P.m, cudaMemcpyDeviceToHost, s));
            M3R_CUDA(cudaMemcpyAsync(P.i2.data(), D.mws.idx2, sizeof(int64_t) * P.m, cudaMemcpyDeviceToHost, s));
            M3R_CUDA(cudaMemcpyAsync(P.c.data(), D.mws.conf, sizeof(float) * P.m, cudaMemcpyDeviceToHost, s));
        }
        M3R_CUDA(cudaStreamSynchronize(s));
    });
    // per phase, the slowest device (the phases end at the all-reduce / the host merge)
    long long total = 0;
    for (int k = 0; k < 4; ++k) phase_ms[k] = 0.0f;
    for (int i = 0; i < nd; ++i) {
        DeviceGuard g(devs_[i]->dev());
        float t[4];
        parts[i].ev->phases(t);
        for (int k = 0; k < 4; ++k) phase_ms[k] = std::max(phase_ms[k], t[k]);
        parts[i].ev.reset();
        total += parts[i].total;
    }
    // merge: all candidates in row order when they fit, else the top_k by (conf desc, idx_1 asc)
    struct C3 {
        float c;
        int64_t i, j;
    };
    std::vector<C3> all;
    for (const Part& P : parts)
        for (int k = 0; k < P.m; ++k) all.push_back({P.c[k], P.i1[k], P.i2[k]});
    if (total > top_k) {
        std::sort(all.begin(), all.end(), [](const C3& a, const C3& b) { return a.c > b.c || (a.c == b.c && a.i < b.i); });
        all.resize(static_cast<size_t>(top_k));
    }
    for (size_t k = 0; k < all.size(); ++k) {
        idx1[k] = all[k].i;
        idx2[k] = all[k].j;
        conf[k] = all[k].c;
    }
    return static_cast<int>(all.size());
}

}  // namespace m3r
