// Bandwidth-bound helper kernels of the two-view model (kernels.cu).  16-bit
// tensors are of the operand type `dt` (DT_F16 or DT_BF16, common.cuh).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace m3r {

// uint8 [n, H, W, 3] -> patch rows [n * (H/p) * (W/p), kpad]; column c*p*p + ky*p + kx,
// value (x/255 - mean_c) / std_c (python_engine.py:176-188), zero in [3*p*p, kpad).
// images [0, na) from img_a, [na, n) from img_b (u8 HWC each); rows of 3 p^2 values padded to kpad
void patch_im2col(cudaStream_t s, int dt, const uint8_t* img_a, const uint8_t* img_b, int na, int n, int H, int W,
                  int p, int kpad, void* out);

// y = LayerNorm(x) * gamma + beta (eps 1e-6), x fp32 [rows, D], y 16-bit [rows, D].
void layernorm(cudaStream_t s, int dt, const float* x, int rows, int D, const float* gamma, const float* beta, void* y);

// fp32 -> 16-bit, n elements (n % 4 == 0).
void cast16(cudaStream_t s, int dt, const float* x, long long n, void* y);

// out[n, H0, W0, C] = f0 + up(f1) + up(f2) + up(f3), bilinear (half-pixel,
// align_corners=False); f_k is [n, h_k, w_k, C], C % 8 == 0.
void dpt_fuse(cudaStream_t s, int dt, const void* f0, const void* f1, int h1, int w1, const void* f2, int h2, int w2,
              const void* f3, int h3, int w3, int n, int H0, int W0, int C, void* out);

// Bilinear resize NHWC [n, hi, wi, C] -> [n, ho, wo, C] (half-pixel), C % 8 == 0.
void resize16(cudaStream_t s, int dt, const void* x, int n, int hi, int wi, int C, int ho, int wo, void* y);

// 3x3 / stride 2 / pad 1 im2col: x [n, h, w, C] -> [n * ho * wo, 9 * C], tap-major.
void im2col_s2(cudaStream_t s, const void* x, int n, int h, int w, int C, void* out);

// out4 fp32 [n, h4, w4, 4] -> pts3d [n, H, W, 3], conf [n, H, W]; bilinear
// (half-pixel) when (h4, w4) != (H, W).
void head_split(cudaStream_t s, const float* out4, int n, int h4, int w4, int H, int W, float* pts3d, float* conf);

// Retrieval attention weights of n_img images of N whitened tokens [N, D] (fp32):
// ||w_r||^2 / (sum_r ||w_r||^2 + 1e-8) (csrc/mps/mpsgraph_engine.mm:843-850).
void retrieval_attention(cudaStream_t s, const float* w, int n_img, int N, int D, float* attn);

// Resize + centre crop of a uint8 [sh, sw, 3] image to [dh, dw, 3], bit-exact with the
// reference's CPU preprocessing (csrc/cpu/preprocessing.cpp:29-63, 84-129).
void resize_crop(cudaStream_t s, const uint8_t* src, int sh, int sw, uint8_t* dst, int dh, int dw);

// The reference CPU head's bilinear resize (backends/python/dpt_head.py:72-116: src = i *
// in / out, no half-pixel offset) of fp32 NHWC maps: [n, hi, wi, C] -> [n, ho, wo, C]
// (C % 4 == 0), and of the 4-channel head output into pts3d [n, ho, wo, 3] + conf [n, ho, wo].
void upsample_ref(cudaStream_t s, const float* x, int n, int hi, int wi, int C, int ho, int wo, float* y);
void upsample_ref_split(cudaStream_t s, const float* x4, int n, int hi, int wi, int ho, int wo, float* pts3d,
                        float* conf);

}  // namespace m3r
