// Host interface of the tcgen05 GEMM (gemm.cuh).  `dt` selects the 16-bit
// operand type (DT_F16 or DT_BF16); operand pointers are 16-bit element arrays.
// cta_pair: 0 = one CTA per 128-row tile, 1 = CTA pairs (256-row tiles, M = 256
// MMAs), -1 = chosen from the problem size.
#pragma once

#include <cuda_runtime.h>

#include "gemm.cuh"
#include "tmap.h"

namespace m3r {

GemmParams gemm_params();

// C = A[M, K] * W[N, K]^T with epilogue `epi`; A and W row-major with row strides
// lda / ldw (elements).  K need not be a multiple of 64 (TMA zero-fills).
void gemm_rows(cudaStream_t s, int dt, int bn, int epi, const void* A, long long lda, int M, int K, const void* W,
               long long ldw, int N, GemmParams p, int cta_pair = -1);

// C = [A0 | A1] * W^T, K = K0 + K1 with K0 % 64 == 0.
void gemm_concat(cudaStream_t s, int dt, int bn, int epi, const void* A0, long long lda0, int K0, const void* A1,
                 long long lda1, int K1, int M, const void* W, long long ldw, int N, GemmParams p,
                 int cta_pair = -1);

// 3x3 convolution, stride 1, pad 1, on NHWC X [n, h, w, c] (pixel stride cstride):
// output pixel rows in NHWC order.  W is [N, 9 * cpad] with cpad = ceil(c / 64) * 64,
// tap-major (ky, kx, channel).
void gemm_conv3(cudaStream_t s, int dt, int bn, int epi, const void* X, int n, int h, int w, int c, int cstride,
                const void* W, int N, GemmParams p, int cta_pair = -1);

int num_sms();

}  // namespace m3r
