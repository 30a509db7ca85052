// ORACLE (test infrastructure only) -- a C entry point over the reference's
// own CPU kernels, compiled from their sources where they lie in the reference
// tree (csrc/cpu/matching.cpp, csrc/cpu/attention.cpp).  Built by
// oracle/Makefile into oracle/_ref/libm3r_ref.so; never part of the product.
//
// The reference declares these functions in no header, so their signatures
// are restated here exactly as they are defined:
//   csrc/cpu/matching.cpp:85-90   mast3r::cpu::reciprocal_match (with and without
//                                 the confidence maps, :110-119)
//   csrc/cpu/matching.cpp:22      mast3r::cpu::normalize_descriptors
//   csrc/cpu/attention.cpp:118    mast3r::cpu::multi_head_attention
// and uses the reference's own Preprocessor class (csrc/cpu/preprocessing.hpp).
#include <cstdint>
#include <cstring>
#include "common/types.hpp"
#include "cpu/preprocessing.hpp"

namespace mast3r {
namespace cpu {
void normalize_descriptors(float* desc, int N, int D);
MatchResult reciprocal_match(const float* desc_1, const float* desc_2,
                             const float* conf_1, const float* conf_2,
                             int height, int width, int desc_dim,
                             const MatchingConfig& config);
void multi_head_attention(const float* Q, const float* K, const float* V, float* output,
                          int B, int H, int N, int D);
}  // namespace cpu
}  // namespace mast3r

extern "C" {

// Runs the reference reciprocal_match on [height*width, d] descriptors.
// Outputs must hold top_k entries.  Returns the match count.
int64_t ref_reciprocal_match(const float* d1, const float* d2, int height, int width, int d,
                             int top_k, int reciprocal, float thr,
                             int64_t* idx1, int64_t* idx2, float* conf,
                             float* pts2d_1, float* pts2d_2) {
    mast3r::MatchingConfig cfg;
    cfg.top_k = top_k;
    cfg.reciprocal = reciprocal != 0;
    cfg.confidence_threshold = thr;
    mast3r::MatchResult r =
        mast3r::cpu::reciprocal_match(d1, d2, nullptr, nullptr, height, width, d, cfg);
    const int64_t n = static_cast<int64_t>(r.num_matches());
    if (n > 0) {
        std::memcpy(idx1, r.idx_1.data(), sizeof(int64_t) * n);
        std::memcpy(idx2, r.idx_2.data(), sizeof(int64_t) * n);
        std::memcpy(conf, r.confidence.data(), sizeof(float) * n);
        std::memcpy(pts2d_1, r.pts2d_1.data(), sizeof(float) * 2 * n);
        std::memcpy(pts2d_2, r.pts2d_2.data(), sizeof(float) * 2 * n);
    }
    return n;
}

// The same with confidence weighting (conf_1, conf_2 [height*width]).
int64_t ref_reciprocal_match_conf(const float* d1, const float* d2, const float* c1, const float* c2, int height,
                                  int width, int d, int top_k, int reciprocal, float thr, int64_t* idx1,
                                  int64_t* idx2, float* conf, float* pts2d_1, float* pts2d_2) {
    mast3r::MatchingConfig cfg;
    cfg.top_k = top_k;
    cfg.reciprocal = reciprocal != 0;
    cfg.confidence_threshold = thr;
    mast3r::MatchResult r = mast3r::cpu::reciprocal_match(d1, d2, c1, c2, height, width, d, cfg);
    const int64_t n = static_cast<int64_t>(r.num_matches());
    if (n > 0) {
        std::memcpy(idx1, r.idx_1.data(), sizeof(int64_t) * n);
        std::memcpy(idx2, r.idx_2.data(), sizeof(int64_t) * n);
        std::memcpy(conf, r.confidence.data(), sizeof(float) * n);
        std::memcpy(pts2d_1, r.pts2d_1.data(), sizeof(float) * 2 * n);
        std::memcpy(pts2d_2, r.pts2d_2.data(), sizeof(float) * 2 * n);
    }
    return n;
}

void ref_normalize(float* desc, int n, int d) { mast3r::cpu::normalize_descriptors(desc, n, d); }

// Preprocessor(res).process: resize + centre crop to res x res, normalise, CHW float.
void ref_preprocess(const uint8_t* img, int h, int w, int res, float* out_chw) {
    mast3r::cpu::Preprocessor p(res);
    mast3r::ImageView v;
    v.data = img;
    v.height = h;
    v.width = w;
    v.channels = 3;
    p.process(v, out_chw);
}

void ref_multi_head_attention(const float* q, const float* k, const float* v, float* o,
                              int b, int h, int n, int d) {
    mast3r::cpu::multi_head_attention(q, k, v, o, b, h, n, d);
}

}  // extern "C"
