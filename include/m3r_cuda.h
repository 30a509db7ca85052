/*
 * m3r_cuda -- C ABI of the B200 (sm_100a) backend for the two-view inference
 * path of mast3r-runtime: engine.infer(img1, img2) and engine.match(desc_1, desc_2).
 *
 * This ABI is what the reference's native-engine slot binds.  The reference's
 * Python dispatcher imports `mast3r_runtime.backends._cuda.CUDAEngine`
 * (mast3r_runtime/backends/__init__.py:173-179), constructs it as
 * CUDAEngine(variant=, resolution=, precision=, num_threads=) (:204-215) and wraps
 * it in NativeEngineWrapper (mast3r_runtime/backends/native_wrapper.py:20-145).
 * The ctypes module mast3r_runtime_b200/_cuda.py implements that object over the
 * functions below.  Each entry point cites the reference interface it replaces.
 *
 * Conventions: every function returns M3R_OK (0) or a negative M3R_ERR_* code;
 * m3r_last_error(engine) / m3r_global_error() give the message.  Buffers are
 * plain host pointers owned by the caller; no pointer is retained after a call
 * returns.  An engine is not re-entrant: calls on one engine must be serialised.
 */
#ifndef M3R_CUDA_H
#define M3R_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define M3R_ABI_VERSION 2

#define M3R_OK 0
#define M3R_ERR_ARG (-1)     /* bad argument, shape or size */
#define M3R_ERR_IO (-2)      /* weights file missing / corrupt / wrong shape */
#define M3R_ERR_CUDA (-3)    /* CUDA runtime or driver error */
#define M3R_ERR_NCCL (-4)    /* NCCL error */
#define M3R_ERR_TIMEOUT (-5) /* a device-side bounded wait ran out */
#define M3R_ERR_STATE (-6)   /* call not valid in the engine's state (e.g. infer before load) */
#define M3R_ERR_NOMEM (-7)   /* device or pinned host allocation failed */

#define M3R_MAX_DEVICES 16

/* 16-bit tensor-core operand type (fp32 accumulation and fp32 residual stream in
 * both).  The reference's precision names map as: "fp16" (its default) and "fp32"
 * -> M3R_DTYPE_F16, "bf16" -> M3R_DTYPE_BF16. */
#define M3R_DTYPE_BF16 0
#define M3R_DTYPE_F16 1

/* Output heads.  M3R_HEAD_MAST3R24: the MASt3R DPT + local-feature head, 24-d
 * L2-normalised descriptors (csrc/mps/mpsgraph_engine.mm:383-437; desc_dim 24).
 * M3R_HEAD_REF_SIMPLE: the reference's CPU head MASt3RDPTHead
 * (mast3r_runtime/backends/python/mast3r_model.py:86-156): 3x3 / 3x3 / 1x1 convs of the
 * first 256 decoder channels at patch-grid resolution, bilinear upsampling
 * (dpt_head.py:72-116), and the first 256 local-feature channels as unnormalised
 * descriptors (desc_dim 256). */
#define M3R_HEAD_MAST3R24 0
#define M3R_HEAD_REF_SIMPLE 1

/* Model architecture + runtime shape.  Dimensions follow the reference's model
 * table (csrc/common/types.hpp:51-69, csrc/mps/graph_builder.hpp:67-77). */
typedef struct m3r_config {
    int patch;      /* 14 (DUNE) or 16 (MASt3R ViT-L) */
    int enc_dim, enc_depth, enc_heads, enc_mlp;
    int dec_dim, dec_depth, dec_heads, dec_mlp;
    int lf_hidden;  /* local-feature MLP width */
    int desc_dim;   /* output descriptor channels: 24 (M3R_HEAD_MAST3R24) or 256 (M3R_HEAD_REF_SIMPLE) */
    int img_h, img_w;   /* input image size, multiples of `patch` */
    int n_devices;      /* 0 = device 0 only */
    int devices[M3R_MAX_DEVICES];
    int max_pairs;      /* image pairs per device per launch (activation buffers) */
    int dtype;          /* M3R_DTYPE_F16 or M3R_DTYPE_BF16 */
    int head;           /* M3R_HEAD_MAST3R24 or M3R_HEAD_REF_SIMPLE */
} m3r_config;

/* Slots of the timing_ms array written by m3r_infer / m3r_match.  m3r_match uses
 * slots 0-2 for its device phases (max over devices): descriptor normalisation, the
 * fused similarity arg-max, and the reciprocal test + threshold + top-k; slot 6 is
 * the three together. */
enum {
    M3R_T_PREPROCESS = 0, /* u8 -> normalised patches (device) */
    M3R_T_ENCODER = 1,
    M3R_T_DECODER = 2,
    M3R_T_HEADS = 3,
    M3R_T_H2D = 4,
    M3R_T_D2H = 5,
    M3R_T_INFERENCE = 6, /* device time of the forward pass / the match (max over devices) */
    M3R_T_TOTAL = 7,     /* host wall time of the call */
    M3R_T_COUNT = 8,
    M3R_T_MATCH_NORMALIZE = 0,
    M3R_T_MATCH_ARGMAX = 1,
    M3R_T_MATCH_SELECT = 2
};

/* Opaque engine: weights replicated on every device of the config. */
typedef struct m3r_engine m3r_engine;

/* ---- module-level queries: replace _cuda.is_available / get_device_name /
 *      get_compute_capability (mast3r_runtime/backends/__init__.py:46-51, 129-138). */
int m3r_version(void);
const char* m3r_global_error(void);
int m3r_device_count(int* count);
int m3r_device_info(int device, char* name, int name_len, int* cc_major, int* cc_minor);

/* ---- engine lifetime: replaces CUDAEngine(variant, resolution, precision, num_threads)
 *      (mast3r_runtime/backends/__init__.py:208-213; reference stub csrc/cuda/bindings.cpp:15-36). */
int m3r_create(const m3r_config* cfg, m3r_engine** out);
void m3r_destroy(m3r_engine* engine);
const char* m3r_last_error(const m3r_engine* engine);

/* ---- load(path): replaces native.load(str(model_path)) (native_wrapper.py:57);
 *      reads a unified safetensors checkpoint in the CroCo key layout. */
int m3r_load(m3r_engine* engine, const char* safetensors_path);
/* is_ready(): native_wrapper.py:45 */
int m3r_is_ready(const m3r_engine* engine);

/* ---- infer(img1, img2): replaces native.infer (native_wrapper.py:84-97).
 * img1, img2: [n_pairs, H, W, 3] uint8.  Outputs (caller-owned, fp32):
 * pts3d_* [n_pairs, H, W, 3], desc_* [n_pairs, H, W, desc_dim], conf_* [n_pairs, H, W].
 * timing_ms: M3R_T_COUNT floats, or NULL.  Pairs are sharded over the devices. */
int m3r_infer(m3r_engine* engine, const uint8_t* img1, const uint8_t* img2, int n_pairs, float* pts3d_1,
              float* pts3d_2, float* desc_1, float* desc_2, float* conf_1, float* conf_2, float* timing_ms);

/* ---- infer(img1, img2) for images of any size: the path the reference's engines take
 * for an image whose size differs from the model's -- aspect-preserving bilinear resize
 * and centre crop (csrc/cpu/preprocessing.cpp:29-63, 84-129; python_engine.py:158-174 with
 * PIL) -- done on the device, bit-exact with the C++ preprocessing, then the forward pass.
 * img1 [h1, w1, 3], img2 [h2, w2, 3] uint8; outputs as m3r_infer for one pair. */
int m3r_infer_any(m3r_engine* engine, const uint8_t* img1, int h1, int w1, const uint8_t* img2, int h2, int w2,
                  float* pts3d_1, float* pts3d_2, float* desc_1, float* desc_2, float* conf_1, float* conf_2,
                  float* timing_ms);

/* ---- retrieval: replaces MPSGraphEngine::load_retrieval / encode_retrieval
 * (csrc/mps/mpsgraph_engine.mm:758-1117, Metal only).  load: a safetensors file with
 * prewhiten.m [enc_dim] and prewhiten.p [enc_dim, enc_dim], after m3r_load (the encoder
 * weights are shared).  encode: images [n_images, H, W, 3] uint8 of the model size ->
 * features [n_images, N, enc_dim] = (encoder output - m) P and attention [n_images, N] =
 * ||feature row||^2 / (sum of them + 1e-8), fp32 (N = patch tokens). */
int m3r_load_retrieval(m3r_engine* engine, const char* safetensors_path);
int m3r_encode_retrieval(m3r_engine* engine, const uint8_t* images, int n_images, float* features, float* attention,
                         float* timing_ms);

/* ---- match(desc_1, desc_2, top_k, reciprocal, confidence_threshold): replaces
 * native.match (native_wrapper.py:122-128) with the semantics of
 * csrc/cpu/matching.cpp:85-237.  desc_*: [height*width, desc_dim] fp32.
 * Outputs hold min(top_k, height*width) entries: idx_* int64, confidence fp32,
 * pts2d_* [n, 2] fp32 (x, y).  With more than top_k matches the result is ordered
 * by confidence descending (idx_1 ascending on ties), otherwise by idx_1.
 * Rows of desc_1 are sharded over the engine's devices. timing_ms as m3r_infer. */
int m3r_match(m3r_engine* engine, const float* desc_1, const float* desc_2, int height, int width, int desc_dim,
              int top_k, int reciprocal, float confidence_threshold, int64_t* idx_1, int64_t* idx_2,
              float* confidence, float* pts2d_1, float* pts2d_2, int* n_matches, float* timing_ms);

/* ---- match(desc_1, desc_2, conf_1, conf_2, pts3d_1, pts3d_2): the full signature of the
 * reference matcher, reciprocal_match(desc_1, desc_2, conf_1, conf_2, pts3d_1, pts3d_2, ...)
 * (mast3r_runtime/backends/matching.py:53-63; csrc/cpu/matching.cpp:85-90).  As m3r_match,
 * plus: conf_1 / conf_2 ([height*width], both or neither) weight every similarity by
 * conf_1[i] * conf_2[j] before the arg-max, threshold and top-k (matching.cpp:110-119);
 * match_pts3d_1 / _2 ([n, 3], both or neither) receive pts3d_1[idx_1] / pts3d_2[idx_2]
 * ([height*width, 3] maps, matching.py:144-152), or zeros when the maps are NULL (the
 * C++ path's result, matching.cpp:231-232). */
int m3r_match_ex(m3r_engine* engine, const float* desc_1, const float* desc_2, const float* conf_1,
                 const float* conf_2, const float* pts3d_1, const float* pts3d_2, int height, int width, int desc_dim,
                 int top_k, int reciprocal, float confidence_threshold, int64_t* idx_1, int64_t* idx_2,
                 float* confidence, float* pts2d_1, float* pts2d_2, float* match_pts3d_1, float* match_pts3d_2,
                 int* n_matches, float* timing_ms);

/* ---- device-resident stages of m3r_infer (throughput measurement and callers that
 * keep outputs on the device): copy inputs in, run, copy outputs out. */
int m3r_stage_inputs(m3r_engine* engine, const uint8_t* img1, const uint8_t* img2, int n_pairs);
int m3r_run_resident(m3r_engine* engine, int n_pairs, float* device_ms);
int m3r_fetch_outputs(m3r_engine* engine, int n_pairs, float* pts3d_1, float* pts3d_2, float* desc_1,
                      float* desc_2, float* conf_1, float* conf_2);

/* Per-kernel-family device time of the last m3r_run_resident / m3r_infer when
 * profiling is on (CUDA events around every launch):
 * out[0] GEMM ms, out[1] GEMM FLOP, out[2] attention ms, out[3] attention FLOP,
 * out[4] other kernels ms, out[5] GEMM launches, out[6] attention launches,
 * out[7] other launches.  Values are for device 0 of the engine. */
int m3r_set_profiling(m3r_engine* engine, int on);

/* Limit (ns) of every bounded device-side wait of the engine's kernels (0 = the default,
 * two seconds).  A kernel whose wait runs out stops, and the call that launched it
 * returns M3R_ERR_TIMEOUT; the CUDA context stays usable.  No reference counterpart:
 * the reference's CUDA backend has no device-side pipeline waits. */
int m3r_set_wait_timeout(m3r_engine* engine, unsigned long long ns);
int m3r_get_profile(const m3r_engine* engine, double* out8);

/* The same profile per operation of the model ("enc.qkv", "enc.attn", "dec.fc2",
 * "head.layer_rn", ...), one line per operation in order of first launch:
 * "<name>\t<ms>\t<flop>\t<launches>\n".  Writes at most cap bytes including the
 * terminating NUL; *needed (when not NULL) gets the full length + 1. */
int m3r_get_profile_ops(const m3r_engine* engine, char* buf, int cap, int* needed);

/* Pinned host memory for zero-staging transfers. */
void* m3r_host_alloc(size_t bytes);
void m3r_host_free(void* p);

/* ---- test / measurement entry points (no reference counterpart; they expose
 * single kernels of this backend for parity tests and kernel timing). ---- */

/* 16-bit operands below are bit patterns of the type `dtype` (M3R_DTYPE_*). */

/* Isolated attention: O[s, t, h*64] = softmax(Q K^T * scale) V, Q [s, h, nq, 64],
 * K/V [s, h, nk, 64].  *kernel_ms gets the mean device time over `iters` launches
 * (>= 1) when not NULL. */
int m3r_attention_fwd(int device, int dtype, const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out,
                      int n_seq, int heads, int nq, int nk, float scale, int iters, float* kernel_ms);

/* GEMM C[M, N] = A[M, K] * W[N, K]^T + bias (16-bit in, fp32 out).  cta_pair: 0 = one
 * CTA per 128-row tile, 1 = CTA pairs (256-row tiles), -1 = chosen from the size. */
int m3r_gemm_test(int device, int dtype, const uint16_t* a, const uint16_t* w, const float* bias, float* c, int M,
                  int N, int K, int bn, int cta_pair, int iters, float* kernel_ms);

/* Residual GEMM as in the transformer blocks' output projections and MLP outputs
 * (backends/python/croco_encoder.py:120-140): c[M, N] += A[M, K] * W[N, K]^T + bias,
 * in place in fp32 (c holds the residual stream on entry).  N a multiple of 4. */
int m3r_gemm_resid_test(int device, int dtype, const uint16_t* a, const uint16_t* w, const float* bias, float* c,
                        int M, int N, int K, int bn, int cta_pair);

/* 3x3 conv, stride 1, pad 1, NHWC: x [n, h, w, c], w [cout, 9 * cpad] (tap-major,
 * channel padded to cpad = ceil(c / 64) * 64) -> y [n, h, w, cout] fp32 (bias added). */
int m3r_conv3_test(int device, int dtype, const uint16_t* x, const uint16_t* w, const float* bias, float* y, int n,
                   int h, int wd, int c, int cout, int bn, int cta_pair);

/* Matcher arg-max only: nn_12 [n1] and nn_21 [n2] (lowest index on ties) of the
 * normalised descriptors, and the row maxima best_12 [n1]. */
int m3r_match_nn(int device, const float* desc_1, const float* desc_2, int64_t n1, int64_t n2, int desc_dim,
                 int32_t* nn_12, int32_t* nn_21, float* best_12, float* kernel_ms);

/* The DPT head's 2x upsampling alone (mpsgraph_engine.mm:402-422, graph_builder.hpp:285-299):
 * x [n, h, w, c] -> y [n, 2h, 2w, c], 16-bit of `dtype`, NHWC, bilinear with half-pixel
 * centres and clamped borders.  c a multiple of 8. */
int m3r_resize2x_test(int device, int dtype, const uint16_t* x, int n, int h, int w, int c, uint16_t* y);

/* The DPT fusion alone (same lines): out [n, H, W, c] = f0 + up(f1) + up(f2) + up(f3), each
 * f_i [n, h_i, w_i, c] upsampled as above to H x W.  c a multiple of 8. */
int m3r_dpt_fuse_test(int device, int dtype, const uint16_t* f0, const uint16_t* f1, int h1, int w1,
                      const uint16_t* f2, int h2, int w2, const uint16_t* f3, int h3, int w3, int n, int H, int W,
                      int c, uint16_t* out);

/* The preprocessing kernel of m3r_infer_any alone: uint8 [h, w, 3] -> [out_h, out_w, 3]. */
int m3r_resize_crop_test(int device, const uint8_t* src, int h, int w, uint8_t* dst, int out_h, int out_w);

/* Self-test of the bounded device waits: a kernel waits on a barrier that nothing
 * signals, with the wait limit limit_ns (0 < limit_ns <= 10 s).  Returns M3R_ERR_TIMEOUT
 * (the expected outcome) with *device_code = the code the wait recorded, after which the
 * device is usable as before.  Errors: m3r_global_error(). */
int m3r_wait_selftest(int device, unsigned long long limit_ns, int* device_code);

/* Validates a checkpoint against a model configuration on the host only (no GPU): every
 * tensor the engine loads is present, F32 / F16 / BF16, with the expected shape, and the
 * file is a well-formed safetensors file.  Returns M3R_OK or M3R_ERR_IO / M3R_ERR_ARG
 * with the reason in m3r_global_error().  Same checks as m3r_load (native_wrapper.py:57
 * loads through it). */
int m3r_check_checkpoint(const m3r_config* cfg, const char* safetensors_path);

/* m3r_match_nn without any device allocation (no counterpart in the reference).
 * For callers that must not allocate GPU memory while running -- a real-time loop
 * that cannot absorb the device synchronisation of cudaMalloc / cudaFree, or a host
 * framework that owns all device memory in its own pool.  Same results as
 * m3r_match_nn, but desc_* (raw, un-normalised) and nn_12 / nn_21 / best_12 are
 * DEVICE buffers on `device`, and the work is queued on `stream` (a cudaStream_t,
 * NULL = default stream) without waiting for it.  Temporaries live in one static
 * 8.25 MiB device array that every GPU loading the library keeps until exit; limits:
 * n1, n2 <= 16384 and desc_dim <= 64 (larger sizes return M3R_ERR_ARG).  The first
 * call on a device looks up the array's address (make it before any stream capture).
 * All calls share the array: calls that overlap on the GPU race.  best_12 may be NULL.
 * Errors: m3r_global_error(). */
int m3r_match_nn_static(int device, const float* desc_1, const float* desc_2, int64_t n1, int64_t n2, int desc_dim,
                        int32_t* nn_12, int32_t* nn_21, float* best_12, void* stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif

#endif /* M3R_CUDA_H */
