// Two-view inference engine: weights replicated per device, one stream and one
// activation arena per device, pairs sharded across devices by host threads.
#pragma once

#include <cuda_runtime.h>

#include <memory>
#include <string>
#include <vector>

#include "../../include/m3r_cuda.h"
#include "matcher.h"

namespace m3r {

struct Dims {
    int patch, enc_dim, enc_depth, enc_heads, enc_mlp;
    int dec_dim, dec_depth, dec_heads, dec_mlp;
    int lf_hidden, desc_dim;  // desc_dim: output descriptor channels (24, or 256 for the reference CPU head)
    int head;                 // M3R_HEAD_MAST3R24 or M3R_HEAD_REF_SIMPLE
    int H, W, hg, wg, ntok;
    int kpad;  // patch-embed K (3 p^2) rounded up to 64
    int hook1, hook2;
    int dt;    // operand type (Dt)
    int dpt_h, dpt_w;  // 16 * grid
    static Dims from(const m3r_config& c);
};

struct Lin {
    uint16_t* w = nullptr;  // [out, in], 16-bit operand type of the engine
    float* b = nullptr;          // [out] or null
    int out = 0, in = 0;
};
struct Norm {
    float* g = nullptr;
    float* b = nullptr;
};
struct EncBlock {
    Norm n1, n2;
    Lin qkv, proj, fc1, fc2;
};
struct DecBlock {
    Norm n1, n2, n3;  // norm_y is folded into kv (Engine::load)
    Lin qkv, proj, q, kv, cproj, fc1, fc2;
};
struct Head {
    Lin ap0_0, ap0_1t, ap1_0, ap1_1t, ap2_0, ap3_0, ap3_1;
    Lin rn[4];
    Lin hd0, hd2;
    float* w4 = nullptr;  // [4][128]
    float* b4 = nullptr;
    Lin lf1, lf2;
};

class Device;

// Optional inputs / outputs of a match: confidence maps that weight every similarity
// (conf_1[i] * conf_2[j], csrc/cpu/matching.cpp:110-119), and 3-D point maps whose
// entries at the matched pixels are returned (matching.py:144-152).  Any may be null.
struct MatchExtras {
    const float* conf_1 = nullptr;   // [n]
    const float* conf_2 = nullptr;   // [n]
    const float* pts3d_1 = nullptr;  // [n, 3]
    const float* pts3d_2 = nullptr;  // [n, 3]
    float* out3_1 = nullptr;         // [<= top_k, 3]
    float* out3_2 = nullptr;
};

class Engine {
public:
    explicit Engine(const m3r_config& cfg);
    ~Engine();
    void load(const std::string& path);
    bool ready() const { return ready_; }
    void infer(const uint8_t* img1, const uint8_t* img2, int n_pairs, float* const outs[6], float* timing);
    // one pair of images of any size, resized and centre-cropped on device 0
    void infer_any(const uint8_t* img1, int h1, int w1, const uint8_t* img2, int h2, int w2, float* const outs[6],
                   float* timing);
    void stage(const uint8_t* img1, const uint8_t* img2, int n_pairs);
    // retrieval: whitening weights, then features + attention weights of k images
    void load_retrieval(const std::string& path);
    void encode_retrieval(const uint8_t* imgs, int k, float* feats, float* attn, float* timing);
    float run_resident(int n_pairs, float* stage_ms);
    void fetch(int n_pairs, float* const outs[6]);
    int match(const float* d1, const float* d2, int h, int w, int d, int top_k, int reciprocal, float thr,
              int64_t* idx1, int64_t* idx2, float* conf, float* p1, float* p2, float* timing,
              const MatchExtras* ex = nullptr);
    void set_profiling(bool on) { profiling_ = on; }
    void set_wait_timeout(unsigned long long ns);  // bounded device waits of every device (0: default)
    void profile(double* out8) const;
    std::string profile_ops() const;  // "<op>\t<ms>\t<flop>\t<launches>\n" per operation

    std::string last_error;
    const Dims& dims() const { return d_; }
    bool profiling() const { return profiling_; }

private:
    std::vector<std::pair<int, int>> shards(int n_pairs) const;  // (first pair, count) per device
    // rows of desc_1 sharded over the devices; column keys max-reduced with NCCL
    int match_multi(const float* d1, const float* d2, const float* c1, const float* c2, long long n, int ww, int dd,
                    int top_k, int reciprocal, float thr, int64_t* idx1, int64_t* idx2, float* conf, float* phase_ms);
    m3r_config cfg_;
    Dims d_;
    std::vector<std::unique_ptr<Device>> devs_;
    std::vector<void*> nccl_comms_;  // ncclComm_t per device, created on the first multi-device match
    bool ready_ = false;
    bool retrieval_ready_ = false;
    bool profiling_ = false;
    int staged_pairs_ = 0;
};

// Reads a checkpoint for the model `d` on the host and discards it: the checks of
// Engine::load without a device (throws Error(kErrIo) / Error(kErrArg)).
void check_checkpoint(const std::string& path, const Dims& d);

// Per-device helpers used by the test entry points.
struct DeviceGuard {
    int prev = 0;
    explicit DeviceGuard(int dev);
    ~DeviceGuard();
};

}  // namespace m3r
