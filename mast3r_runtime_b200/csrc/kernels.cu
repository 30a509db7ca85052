// Bandwidth-bound helper kernels: vectorised (16-byte) loads and stores,
// grid-stride loops with grids capped at a multiple of the SM count.
#include "common.cuh"
#include "kernels.h"
#include "tmap.h"

namespace m3r {

namespace {

inline int grid_for(long long n, int block) {
    long long g = (n + block - 1) / block;
    if (g > 148LL * 32) g = 148LL * 32;
    return static_cast<int>(g > 0 ? g : 1);
}

template <class T>
__global__ void patch_im2col_kernel(const uint8_t* __restrict__ img_a, const uint8_t* __restrict__ img_b, int na,
                                    int n, int H, int W, int p, int kpad, T* __restrict__ out) {
    const int hg = H / p, wg = W / p;
    const long long total = static_cast<long long>(n) * hg * wg * kpad;
    const float mean[3] = {0.485f, 0.456f, 0.406f};
    const float stdv[3] = {0.229f, 0.224f, 0.225f};
    for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < total;
         e += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int k = static_cast<int>(e % kpad);
        const long long row = e / kpad;
        float v = 0.0f;
        if (k < 3 * p * p) {
            const int c = k / (p * p);
            const int rem = k - c * p * p;
            const int ky = rem / p, kx = rem - (rem / p) * p;
            const int im = static_cast<int>(row / (hg * wg));
            const int t = static_cast<int>(row - static_cast<long long>(im) * hg * wg);
            const int gy = t / wg, gx = t - (t / wg) * wg;
            const uint8_t* img = im < na ? img_a + static_cast<long long>(im) * H * W * 3
                                         : img_b + static_cast<long long>(im - na) * H * W * 3;
            const uint8_t u = img[(static_cast<long long>(gy * p + ky) * W + gx * p + kx) * 3 + c];
            v = (static_cast<float>(u) / 255.0f - mean[c]) / stdv[c];
        }
        out[e] = Elem<T>::from(v);
    }
}

// One warp per row; two-pass mean / variance in fp32 (vit_encoder.py:98-108).
template <class T>
__global__ void layernorm_kernel(const float* __restrict__ x, int rows, int D, const float* __restrict__ g,
                                 const float* __restrict__ b, T* __restrict__ y) {
    const int warps = blockDim.x >> 5;
    const int lane = threadIdx.x & 31;
    for (long long r = static_cast<long long>(blockIdx.x) * warps + (threadIdx.x >> 5); r < rows;
         r += static_cast<long long>(gridDim.x) * warps) {
        const float4* xr = reinterpret_cast<const float4*>(x + r * D);
        const int n4 = D >> 2;
        float4 v[8];  // D <= 1024
        float s = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int idx = lane + 32 * i;
            if (idx < n4) {
                v[i] = xr[idx];
                s += v[i].x + v[i].y + v[i].z + v[i].w;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        const float mean = s / D;
        float q = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int idx = lane + 32 * i;
            if (idx < n4) {
                const float a = v[i].x - mean, bb = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
                q += a * a + bb * bb + c * c + d * d;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
        const float rstd = rsqrtf(q / D + 1e-6f);
        uint2* yr = reinterpret_cast<uint2*>(y + r * D);
        const float4* g4 = reinterpret_cast<const float4*>(g);
        const float4* b4 = reinterpret_cast<const float4*>(b);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int idx = lane + 32 * i;
            if (idx < n4) {
                const float4 gg = __ldg(g4 + idx), bb = __ldg(b4 + idx);
                uint2 u;
                u.x = Elem<T>::pack((v[i].x - mean) * rstd * gg.x + bb.x, (v[i].y - mean) * rstd * gg.y + bb.y);
                u.y = Elem<T>::pack((v[i].z - mean) * rstd * gg.z + bb.z, (v[i].w - mean) * rstd * gg.w + bb.w);
                yr[idx] = u;
            }
        }
    }
}

template <class T>
__global__ void cast16_kernel(const float* __restrict__ x, long long n, T* __restrict__ y) {
    const long long n4 = n >> 2;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const float4 v = reinterpret_cast<const float4*>(x)[i];
        uint2 u;
        u.x = Elem<T>::pack(v.x, v.y);
        u.y = Elem<T>::pack(v.z, v.w);
        reinterpret_cast<uint2*>(y)[i] = u;
    }
}

// half-pixel source coordinate, clamped like PyTorch / MPSGraph (align_corners=False)
__device__ __forceinline__ void src_coord(int o, int n_in, int n_out, int& i0, int& i1, float& f) {
    float s = (o + 0.5f) * (static_cast<float>(n_in) / n_out) - 0.5f;
    s = fmaxf(s, 0.0f);
    i0 = min(static_cast<int>(s), n_in - 1);
    i1 = min(i0 + 1, n_in - 1);
    f = s - i0;
}

struct F8 {
    float v[8];
};

template <class T>
__device__ __forceinline__ void load8(const T* p, F8& o) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t* w = reinterpret_cast<const uint32_t*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = Elem<T>::unpack(w[i]);
        o.v[2 * i] = f.x;
        o.v[2 * i + 1] = f.y;
    }
}

template <class T>
__device__ __forceinline__ void store8(T* p, const F8& o) {
    uint4 u;
    uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = Elem<T>::pack(o.v[2 * i], o.v[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = u;
}

template <class T>
__device__ __forceinline__ void bilerp_acc(const T* base, int hi, int wi, int C, int Ho, int Wo, int y, int x, int c8,
                                           F8& acc) {
    int y0, y1, x0, x1;
    float fy, fx;
    src_coord(y, hi, Ho, y0, y1, fy);
    src_coord(x, wi, Wo, x0, x1, fx);
    F8 a, b, c, d;
    load8(base + (static_cast<long long>(y0) * wi + x0) * C + c8, a);
    load8(base + (static_cast<long long>(y0) * wi + x1) * C + c8, b);
    load8(base + (static_cast<long long>(y1) * wi + x0) * C + c8, c);
    load8(base + (static_cast<long long>(y1) * wi + x1) * C + c8, d);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float top = a.v[i] * (1.0f - fx) + b.v[i] * fx;
        const float bot = c.v[i] * (1.0f - fx) + d.v[i] * fx;
        acc.v[i] += top * (1.0f - fy) + bot * fy;
    }
}

// Mixed-precision multiply-add (sm_100 fma.rn.f32.{f16,bf16}): d = a * w + c with 16-bit a
// and w of the operand type T, fp32 c and d, one rounding.  Interpolation weights that are
// multiples of 1/256 (the 2x / 4x / 8x half-pixel fractions and their products) are exact in
// both 16-bit types and their products with a 16-bit value exact in fp32, so the
// interpolations below need no 16 -> 32-bit conversions and round once per term.
template <class T>
struct Mix;
template <>
struct Mix<__half> {
    // (d0, d1) = (lo(pair), hi(pair)) * w + (c0, c1)
    __device__ static __forceinline__ void fma2(uint32_t pair, uint16_t w, float c0, float c1, float& d0, float& d1) {
        asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
            "fma.rn.f32.f16 %0, lo, %3, %4;\n\tfma.rn.f32.f16 %1, hi, %3, %5;\n\t}"
            : "=f"(d0), "=f"(d1)
            : "r"(pair), "h"(w), "f"(c0), "f"(c1));
    }
    __device__ static __forceinline__ uint16_t bits(float w) { return __half_as_ushort(__float2half_rn(w)); }
};
template <>
struct Mix<__nv_bfloat16> {
    __device__ static __forceinline__ void fma2(uint32_t pair, uint16_t w, float c0, float c1, float& d0, float& d1) {
        asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
            "fma.rn.f32.bf16 %0, lo, %3, %4;\n\tfma.rn.f32.bf16 %1, hi, %3, %5;\n\t}"
            : "=f"(d0), "=f"(d1)
            : "r"(pair), "h"(w), "f"(c0), "f"(c1));
    }
    __device__ static __forceinline__ uint16_t bits(float w) {
        return __bfloat16_as_ushort(__float2bfloat16_rn(w));
    }
};

__device__ __forceinline__ uint4 ld16(const void* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ uint32_t word(const uint4& u, int q) {
    return q == 0 ? u.x : q == 1 ? u.y : q == 2 ? u.z : u.w;
}

// acc += bilinear sample (half-pixel centres, clamped) of an 8-channel chunk, weights
// w00..w11 in the operand type (exact for the power-of-two ratios it is used with)
template <class T>
__device__ __forceinline__ void bilerp_mix(const T* base, int hi, int wi, int C, int Ho, int Wo, int y, int x, int c8,
                                           float (&acc)[8]) {
    int y0, y1, x0, x1;
    float fy, fx;
    src_coord(y, hi, Ho, y0, y1, fy);
    src_coord(x, wi, Wo, x0, x1, fx);
    const uint16_t w00 = Mix<T>::bits((1.0f - fx) * (1.0f - fy)), w01 = Mix<T>::bits(fx * (1.0f - fy));
    const uint16_t w10 = Mix<T>::bits((1.0f - fx) * fy), w11 = Mix<T>::bits(fx * fy);
    const uint4 a = ld16(base + (static_cast<long long>(y0) * wi + x0) * C + c8);
    const uint4 b = ld16(base + (static_cast<long long>(y0) * wi + x1) * C + c8);
    const uint4 c = ld16(base + (static_cast<long long>(y1) * wi + x0) * C + c8);
    const uint4 d = ld16(base + (static_cast<long long>(y1) * wi + x1) * C + c8);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        float& s0 = acc[2 * q];
        float& s1 = acc[2 * q + 1];
        Mix<T>::fma2(word(a, q), w00, s0, s1, s0, s1);
        Mix<T>::fma2(word(b, q), w01, s0, s1, s0, s1);
        Mix<T>::fma2(word(c, q), w10, s0, s1, s0, s1);
        Mix<T>::fma2(word(d, q), w11, s0, s1, s0, s1);
    }
}

// Grid of the NHWC elementwise kernels below: blockIdx.z = image, blockIdx.y =
// (output) row, x = (pixel in the row, 8-channel chunk); no 64-bit division.
struct RowGrid {
    int c8n;  // 8-channel chunks per pixel
    __device__ __forceinline__ bool at(int w, int& x, int& c8) const {
        const int e = blockIdx.x * blockDim.x + threadIdx.x;
        x = e / c8n;
        c8 = (e - x * c8n) * 8;
        return x < w;
    }
};

inline dim3 row_grid(int n, int rows, int w, int c8n, int block) {
    return dim3((w * c8n + block - 1) / block, rows, n);
}

template <class T>
__global__ void dpt_fuse_kernel(const T* __restrict__ f0, const T* __restrict__ f1, int h1, int w1,
                                const T* __restrict__ f2, int h2, int w2, const T* __restrict__ f3, int h3, int w3,
                                int H0, int W0, int C, T* __restrict__ out) {
    int x, c8;
    if (!RowGrid{C / 8}.at(W0, x, c8)) return;
    const int y = blockIdx.y;
    const long long im = blockIdx.z;
    F8 acc;
    load8(f0 + ((im * H0 + y) * W0 + x) * C + c8, acc);
    bilerp_acc(f1 + im * h1 * w1 * C, h1, w1, C, H0, W0, y, x, c8, acc);
    bilerp_acc(f2 + im * h2 * w2 * C, h2, w2, C, H0, W0, y, x, c8, acc);
    bilerp_acc(f3 + im * h3 * w3 * C, h3, w3, C, H0, W0, y, x, c8, acc);
    store8(out + ((im * H0 + y) * W0 + x) * C + c8, acc);
}

// dpt_fuse_kernel for levels at exactly 1/2, 1/4 and 1/8 of the output size (the DPT
// pyramid of every model size here): mixed-precision accumulation, no conversions.
template <class T>
__global__ void dpt_fuse_pow2_kernel(const T* __restrict__ f0, const T* __restrict__ f1, const T* __restrict__ f2,
                                     const T* __restrict__ f3, int H0, int W0, int C, T* __restrict__ out) {
    int x, c8;
    if (!RowGrid{C / 8}.at(W0, x, c8)) return;
    const int y = blockIdx.y;
    const long long im = blockIdx.z;
    float acc[8];
    const uint4 u = ld16(f0 + ((im * H0 + y) * W0 + x) * C + c8);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float2 f = Elem<T>::unpack(word(u, q));
        acc[2 * q] = f.x;
        acc[2 * q + 1] = f.y;
    }
    const int h1 = H0 / 2, w1 = W0 / 2, h2 = H0 / 4, w2 = W0 / 4, h3 = H0 / 8, w3 = W0 / 8;
    bilerp_mix(f1 + im * h1 * w1 * C, h1, w1, C, H0, W0, y, x, c8, acc);
    bilerp_mix(f2 + im * h2 * w2 * C, h2, w2, C, H0, W0, y, x, c8, acc);
    bilerp_mix(f3 + im * h3 * w3 * C, h3, w3, C, H0, W0, y, x, c8, acc);
    uint4 o;
    o.x = Elem<T>::pack(acc[0], acc[1]);
    o.y = Elem<T>::pack(acc[2], acc[3]);
    o.z = Elem<T>::pack(acc[4], acc[5]);
    o.w = Elem<T>::pack(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + ((im * H0 + y) * W0 + x) * C + c8) = o;
}

template <class T>
__global__ void resize_kernel(const T* __restrict__ x, int hi, int wi, int C, int ho, int wo, T* __restrict__ y) {
    int ox, c8;
    if (!RowGrid{C / 8}.at(wo, ox, c8)) return;
    const int oy = blockIdx.y;
    const long long im = blockIdx.z;
    F8 acc;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc.v[i] = 0.0f;
    bilerp_acc(x + im * hi * wi * C, hi, wi, C, ho, wo, oy, ox, c8, acc);
    store8(y + ((im * ho + oy) * wo + ox) * C + c8, acc);
}

// Exact 2x upsampling (half-pixel centres): output row 2i takes input rows i-1, i
// with weights 0.25, 0.75 and row 2i+1 takes i, i+1 with 0.75, 0.25, the
// neighbours clamped at the borders (which reproduces the clamped source
// coordinate of bilerp_acc); the same along x.  A thread owns one 8-channel chunk of
// input column ix over kResizeRows input rows: it keeps the x-interpolated values of
// rows iy-1, iy, iy+1 in registers (a sliding window, three 16-byte loads per input
// row) and writes the four output pixels (2iy + a, 2ix + b) of each row.
constexpr int kResizeRows = 4;

// (o0, o1) = 0.75 * (c0, c1) + 0.25 * (e0, e1) in two packed fp32 operations
__device__ __forceinline__ void lerp_q2(float c0, float c1, float e0, float e1, float& o0, float& o1) {
    asm("{\n\t.reg .b64 c, e, k1, k3, t;\n\t"
        "mov.b64 c, {%2, %3};\n\tmov.b64 e, {%4, %5};\n\t"
        "mov.b64 k1, {%6, %6};\n\tmov.b64 k3, {%7, %7};\n\t"
        "mul.rn.f32x2 t, e, k1;\n\tfma.rn.f32x2 t, c, k3, t;\n\t"
        "mov.b64 {%0, %1}, t;\n\t}"
        : "=f"(o0), "=f"(o1)
        : "f"(c0), "f"(c1), "f"(e0), "f"(e1), "f"(0.25f), "f"(0.75f));
}

// x-interpolation of one input row at column ix: h[b][i] = output column 2ix + b
template <class T>
__device__ __forceinline__ void resize2x_row(const T* row, int C, int xl, int xc, int xr, uint16_t q1, uint16_t q3,
                                             float (&h)[2][8]) {
    const uint4 l = ld16(row + static_cast<long long>(xl) * C);
    const uint4 m = ld16(row + static_cast<long long>(xc) * C);
    const uint4 r = ld16(row + static_cast<long long>(xr) * C);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        float t0, t1;
        Mix<T>::fma2(word(m, q), q3, 0.0f, 0.0f, t0, t1);  // 0.75 * centre: exact in fp32
        Mix<T>::fma2(word(l, q), q1, t0, t1, h[0][2 * q], h[0][2 * q + 1]);
        Mix<T>::fma2(word(r, q), q1, t0, t1, h[1][2 * q], h[1][2 * q + 1]);
    }
}

template <class T>
__global__ void resize2x_kernel(const T* __restrict__ x, int hi, int wi, int C, T* __restrict__ y) {
    int ix, c8;
    if (!RowGrid{C / 8}.at(wi, ix, c8)) return;
    const int iy0 = blockIdx.y * kResizeRows;
    const long long im = blockIdx.z;
    const T* base = x + im * hi * wi * C + c8;
    const int ho = 2 * hi, wo = 2 * wi;
    const int xl = max(ix - 1, 0), xr = min(ix + 1, wi - 1);
    const uint16_t q1 = Mix<T>::bits(0.25f), q3 = Mix<T>::bits(0.75f);
    float hp[2][8], hc[2][8], hn[2][8];  // rows iy - 1, iy, iy + 1 (clamped)
    resize2x_row(base + static_cast<long long>(max(iy0 - 1, 0)) * wi * C, C, xl, ix, xr, q1, q3, hp);
    resize2x_row(base + static_cast<long long>(iy0) * wi * C, C, xl, ix, xr, q1, q3, hc);
#pragma unroll
    for (int k = 0; k < kResizeRows; ++k) {
        const int iy = iy0 + k;
        if (iy >= hi) break;
        resize2x_row(base + static_cast<long long>(min(iy + 1, hi - 1)) * wi * C, C, xl, ix, xr, q1, q3, hn);
#pragma unroll
        for (int a = 0; a < 2; ++a) {
#pragma unroll
            for (int b = 0; b < 2; ++b) {
                // row 2iy: 0.75 row iy + 0.25 row iy-1; row 2iy + 1: 0.75 row iy + 0.25 row iy+1
                const float(&e)[2][8] = a == 0 ? hp : hn;
                float o[8];
#pragma unroll
                for (int i = 0; i < 8; i += 2) lerp_q2(hc[b][i], hc[b][i + 1], e[b][i], e[b][i + 1], o[i], o[i + 1]);
                uint4 u;
                u.x = Elem<T>::pack(o[0], o[1]);
                u.y = Elem<T>::pack(o[2], o[3]);
                u.z = Elem<T>::pack(o[4], o[5]);
                u.w = Elem<T>::pack(o[6], o[7]);
                *reinterpret_cast<uint4*>(y + ((im * ho + 2 * iy + a) * wo + 2 * ix + b) * C + c8) = u;
            }
        }
#pragma unroll
        for (int b = 0; b < 2; ++b)
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                hp[b][i] = hc[b][i];
                hc[b][i] = hn[b][i];
            }
    }
}

// 16-bit agnostic: moves 8-element (16-byte) chunks
__global__ void im2col_s2_kernel(const uint16_t* __restrict__ x, int n, int h, int w, int C,
                                 uint16_t* __restrict__ out) {
    const int ho = (h - 1) / 2 + 1, wo = (w - 1) / 2 + 1;
    const int c8n = C / 8;
    const long long total = static_cast<long long>(n) * ho * wo * 9 * c8n;
    for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < total;
         e += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int c8 = static_cast<int>(e % c8n) * 8;
        long long r = e / c8n;
        const int tap = static_cast<int>(r % 9);
        r /= 9;
        const int xo = static_cast<int>(r % wo);
        r /= wo;
        const int yo = static_cast<int>(r % ho);
        const int im = static_cast<int>(r / ho);
        const int yi = 2 * yo + tap / 3 - 1, xi = 2 * xo + tap % 3 - 1;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (yi >= 0 && yi < h && xi >= 0 && xi < w)
            v = *reinterpret_cast<const uint4*>(x + ((static_cast<long long>(im) * h + yi) * w + xi) * C + c8);
        *reinterpret_cast<uint4*>(out + e * 8) = v;
    }
}

// Resize + centre crop of a uint8 RGB image to the model size, bit-exact with the
// reference's CPU preprocessing (csrc/cpu/preprocessing.cpp:29-63, 84-129): scale =
// max(dh / sh, dw / sw), new = (int)(s * scale), bilinear resize to new (src = d * s / new,
// truncated, clamped neighbours), crop [(new - d) / 2, +d); every multiply and add
// separately rounded, the weighted sum clamped to [0, 255] and truncated.  Rows / columns
// the reference would read past its resized buffer (new < d after truncation) are
// clamped to the last one.  One thread per output pixel.
__global__ void resize_crop_kernel(const uint8_t* __restrict__ src, int sh, int sw, uint8_t* __restrict__ dst, int dh,
                                   int dw, int new_h, int new_w, float scale_y, float scale_x) {
    const long long total = static_cast<long long>(dh) * dw;
    const int start_h = (new_h - dh) / 2, start_w = (new_w - dw) / 2;
    for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < total;
         e += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int x = static_cast<int>(e % dw), y = static_cast<int>(e / dw);
        const int ry = min(start_h + y, new_h - 1), rx = min(start_w + x, new_w - 1);
        const float syf = __fmul_rn(static_cast<float>(ry), scale_y);
        const float sxf = __fmul_rn(static_cast<float>(rx), scale_x);
        const int y0 = static_cast<int>(syf), x0 = static_cast<int>(sxf);
        const int y1 = min(y0 + 1, sh - 1), x1 = min(x0 + 1, sw - 1);
        const float fy = __fsub_rn(syf, static_cast<float>(y0)), fx = __fsub_rn(sxf, static_cast<float>(x0));
        const float gy = __fsub_rn(1.0f, fy), gx = __fsub_rn(1.0f, fx);
        const float w00 = __fmul_rn(gx, gy), w01 = __fmul_rn(fx, gy), w10 = __fmul_rn(gx, fy), w11 = __fmul_rn(fx, fy);
        const uint8_t* p00 = src + (static_cast<long long>(y0) * sw + x0) * 3;
        const uint8_t* p01 = src + (static_cast<long long>(y0) * sw + x1) * 3;
        const uint8_t* p10 = src + (static_cast<long long>(y1) * sw + x0) * 3;
        const uint8_t* p11 = src + (static_cast<long long>(y1) * sw + x1) * 3;
        uint8_t* o = dst + e * 3;
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            float v = __fmul_rn(w00, static_cast<float>(p00[c]));
            v = __fadd_rn(v, __fmul_rn(w01, static_cast<float>(p01[c])));
            v = __fadd_rn(v, __fmul_rn(w10, static_cast<float>(p10[c])));
            v = __fadd_rn(v, __fmul_rn(w11, static_cast<float>(p11[c])));
            v = fminf(fmaxf(v, 0.0f), 255.0f);
            o[c] = static_cast<uint8_t>(v);
        }
    }
}

// Retrieval attention weights (csrc/mps/mpsgraph_engine.mm:843-850): per image of N
// whitened tokens w [N, D], a[r] = ||w_r||^2 / (sum_r ||w_r||^2 + 1e-8).  One block per
// image; a warp per row for the squared norms, then a block sum.
__global__ void retrieval_attention_kernel(const float* __restrict__ w, int N, int D, float* __restrict__ attn) {
    __shared__ float s_part[32];
    __shared__ float s_total;
    const int img = blockIdx.x;
    const float* base = w + static_cast<long long>(img) * N * D;
    float* a = attn + static_cast<long long>(img) * N;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    float local = 0.0f;
    for (int r = warp; r < N; r += nw) {
        const float* row = base + static_cast<long long>(r) * D;
        float acc = 0.0f;
        for (int c = lane; c < D; c += 32) acc += row[c] * row[c];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) a[r] = acc;
        local += acc;
    }
    if (lane == 0) s_part[warp] = local;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int i = 0; i < nw; ++i) t += s_part[i];
        s_total = t + 1e-8f;
    }
    __syncthreads();
    const float inv_total = s_total;
    for (int r = threadIdx.x; r < N; r += blockDim.x) a[r] = a[r] / inv_total;
}

// Source rows / columns of output index i under the reference CPU head's bilinear
// resize (backends/python/dpt_head.py:72-116): src = i * in / out (no half-pixel
// offset), i0 = floor(src), i1 = min(i0 + 1, in - 1), f = src - i0; the rational src
// is formed exactly in integers.
__device__ __forceinline__ void ref_coord(int i, int in, int out, int& i0, int& i1, float& f) {
    const long long num = static_cast<long long>(i) * in;
    i0 = static_cast<int>(num / out);
    f = static_cast<float>(num - static_cast<long long>(i0) * out) / static_cast<float>(out);
    i1 = min(i0 + 1, in - 1);
}

// the four-term blend in the reference's order: (1-fh)(1-fw) a + (1-fh) fw b + fh (1-fw) c + fh fw d
__device__ __forceinline__ float ref_blend(float a, float b, float c, float d, float fh, float fw) {
    return (1.0f - fh) * (1.0f - fw) * a + (1.0f - fh) * fw * b + fh * (1.0f - fw) * c + fh * fw * d;
}

// [n, hi, wi, C] fp32 -> [n, ho, wo, C] fp32, four channels per thread (C % 4 == 0)
__global__ void upsample_ref_kernel(const float4* __restrict__ x, int n, int hi, int wi, int C4, int ho, int wo,
                                    float4* __restrict__ y) {
    const long long total = static_cast<long long>(n) * ho * wo * C4;
    for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < total;
         e += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(e % C4);
        const long long pix = e / C4;
        const int ox = static_cast<int>(pix % wo);
        const int oy = static_cast<int>((pix / wo) % ho);
        const int im = static_cast<int>(pix / (static_cast<long long>(wo) * ho));
        int y0, y1, x0, x1;
        float fh, fw;
        ref_coord(oy, hi, ho, y0, y1, fh);
        ref_coord(ox, wi, wo, x0, x1, fw);
        const float4* base = x + static_cast<long long>(im) * hi * wi * C4 + c;
        const float4 a = base[(static_cast<long long>(y0) * wi + x0) * C4], b = base[(static_cast<long long>(y0) * wi + x1) * C4];
        const float4 q = base[(static_cast<long long>(y1) * wi + x0) * C4], d = base[(static_cast<long long>(y1) * wi + x1) * C4];
        y[e] = make_float4(ref_blend(a.x, b.x, q.x, d.x, fh, fw), ref_blend(a.y, b.y, q.y, d.y, fh, fw),
                           ref_blend(a.z, b.z, q.z, d.z, fh, fw), ref_blend(a.w, b.w, q.w, d.w, fh, fw));
    }
}

// [n, hi, wi, 4] fp32 (pts3d xyz, confidence) -> pts3d [n, ho, wo, 3], conf [n, ho, wo]
__global__ void upsample_ref_split_kernel(const float4* __restrict__ x, int n, int hi, int wi, int ho, int wo,
                                          float* __restrict__ pts, float* __restrict__ conf) {
    const long long total = static_cast<long long>(n) * ho * wo;
    for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < total;
         e += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int ox = static_cast<int>(e % wo);
        const int oy = static_cast<int>((e / wo) % ho);
        const int im = static_cast<int>(e / (static_cast<long long>(wo) * ho));
        int y0, y1, x0, x1;
        float fh, fw;
        ref_coord(oy, hi, ho, y0, y1, fh);
        ref_coord(ox, wi, wo, x0, x1, fw);
        const float4* base = x + static_cast<long long>(im) * hi * wi;
        const float4 a = base[y0 * wi + x0], b = base[y0 * wi + x1], q = base[y1 * wi + x0], d = base[y1 * wi + x1];
        pts[e * 3 + 0] = ref_blend(a.x, b.x, q.x, d.x, fh, fw);
        pts[e * 3 + 1] = ref_blend(a.y, b.y, q.y, d.y, fh, fw);
        pts[e * 3 + 2] = ref_blend(a.z, b.z, q.z, d.z, fh, fw);
        conf[e] = ref_blend(a.w, b.w, q.w, d.w, fh, fw);
    }
}

__global__ void head_split_kernel(const float* __restrict__ o4, int n, int h4, int w4, int H, int W,
                                  float* __restrict__ pts, float* __restrict__ conf) {
    const long long total = static_cast<long long>(n) * H * W;
    for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < total;
         e += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int x = static_cast<int>(e % W);
        const int y = static_cast<int>((e / W) % H);
        const int im = static_cast<int>(e / (static_cast<long long>(W) * H));
        const float4* base = reinterpret_cast<const float4*>(o4) + static_cast<long long>(im) * h4 * w4;
        float4 v;
        if (h4 == H && w4 == W) {
            v = base[static_cast<long long>(y) * w4 + x];
        } else {
            int y0, y1, x0, x1;
            float fy, fx;
            src_coord(y, h4, H, y0, y1, fy);
            src_coord(x, w4, W, x0, x1, fx);
            const float4 a = base[y0 * w4 + x0], b = base[y0 * w4 + x1], c = base[y1 * w4 + x0],
                         d = base[y1 * w4 + x1];
            auto lerp2 = [&](float pa, float pb, float pc, float pd) {
                return (pa * (1.0f - fx) + pb * fx) * (1.0f - fy) + (pc * (1.0f - fx) + pd * fx) * fy;
            };
            v = make_float4(lerp2(a.x, b.x, c.x, d.x), lerp2(a.y, b.y, c.y, d.y), lerp2(a.z, b.z, c.z, d.z),
                            lerp2(a.w, b.w, c.w, d.w));
        }
        pts[e * 3 + 0] = v.x;
        pts[e * 3 + 1] = v.y;
        pts[e * 3 + 2] = v.z;
        conf[e] = v.w;
    }
}

#define M3R_BY_DT(dt, ...)                                                  \
    do {                                                                    \
        if ((dt) == DT_F16) {                                               \
            using T = __half;                                               \
            __VA_ARGS__;                                                    \
        } else if ((dt) == DT_BF16) {                                       \
            using T = __nv_bfloat16;                                        \
            __VA_ARGS__;                                                    \
        } else {                                                            \
            throw Error(kErrArg, "unknown operand type");                   \
        }                                                                   \
    } while (0)

}  // namespace

void patch_im2col(cudaStream_t s, int dt, const uint8_t* img_a, const uint8_t* img_b, int na, int n, int H, int W,
                  int p, int kpad, void* out) {
    const long long total = static_cast<long long>(n) * (H / p) * (W / p) * kpad;
    M3R_BY_DT(dt, patch_im2col_kernel<T><<<grid_for(total, 256), 256, 0, s>>>(img_a, img_b, na, n, H, W, p, kpad,
                                                                                  static_cast<T*>(out)));
    M3R_CUDA(cudaGetLastError());
}

void layernorm(cudaStream_t s, int dt, const float* x, int rows, int D, const float* gamma, const float* beta, void* y) {
    M3R_REQUIRE(D % 4 == 0 && D <= 1024, "layernorm: D must be a multiple of 4 and <= 1024");
    if (rows == 0) return;
    const int warps = 8;
    long long blocks = (rows + warps - 1) / warps;
    if (blocks > 148LL * 16) blocks = 148LL * 16;
    M3R_BY_DT(dt, layernorm_kernel<T><<<static_cast<int>(blocks), warps * 32, 0, s>>>(x, rows, D, gamma, beta, static_cast<T*>(y)));
    M3R_CUDA(cudaGetLastError());
}

void cast16(cudaStream_t s, int dt, const float* x, long long n, void* y) {
    M3R_REQUIRE(n % 4 == 0, "cast16: size must be a multiple of 4");
    M3R_BY_DT(dt, cast16_kernel<T><<<grid_for(n / 4, 256), 256, 0, s>>>(x, n, static_cast<T*>(y)));
    M3R_CUDA(cudaGetLastError());
}

void dpt_fuse(cudaStream_t s, int dt, const void* f0, const void* f1, int h1, int w1, const void* f2, int h2, int w2,
              const void* f3, int h3, int w3, int n, int H0, int W0, int C, void* out) {
    M3R_REQUIRE(C % 8 == 0, "dpt_fuse: C % 8");
    M3R_REQUIRE(n <= 65535 && H0 <= 65535, "dpt_fuse: grid too large");
    if (H0 == 2 * h1 && W0 == 2 * w1 && H0 == 4 * h2 && W0 == 4 * w2 && H0 == 8 * h3 && W0 == 8 * w3) {
        M3R_BY_DT(dt, dpt_fuse_pow2_kernel<T><<<row_grid(n, H0, W0, C / 8, 128), 128, 0, s>>>(
                          static_cast<const T*>(f0), static_cast<const T*>(f1), static_cast<const T*>(f2),
                          static_cast<const T*>(f3), H0, W0, C, static_cast<T*>(out)));
    } else {
        M3R_BY_DT(dt, dpt_fuse_kernel<T><<<row_grid(n, H0, W0, C / 8, 128), 128, 0, s>>>(
                          static_cast<const T*>(f0), static_cast<const T*>(f1), h1, w1, static_cast<const T*>(f2), h2,
                          w2, static_cast<const T*>(f3), h3, w3, H0, W0, C, static_cast<T*>(out)));
    }
    M3R_CUDA(cudaGetLastError());
}

void resize16(cudaStream_t s, int dt, const void* x, int n, int hi, int wi, int C, int ho, int wo, void* y) {
    M3R_REQUIRE(C % 8 == 0, "resize16: C % 8");
    M3R_REQUIRE(n <= 65535 && ho <= 65535, "resize16: grid too large");
    if (ho == 2 * hi && wo == 2 * wi) {
        M3R_BY_DT(dt, resize2x_kernel<T><<<row_grid(n, (hi + kResizeRows - 1) / kResizeRows, wi, C / 8, 128), 128, 0,
                                           s>>>(
                          static_cast<const T*>(x), hi, wi, C, static_cast<T*>(y)));
    } else {
        M3R_BY_DT(dt, resize_kernel<T><<<row_grid(n, ho, wo, C / 8, 128), 128, 0, s>>>(
                          static_cast<const T*>(x), hi, wi, C, ho, wo, static_cast<T*>(y)));
    }
    M3R_CUDA(cudaGetLastError());
}

void im2col_s2(cudaStream_t s, const void* x, int n, int h, int w, int C, void* out) {
    M3R_REQUIRE(C % 8 == 0, "im2col_s2: C % 8");
    const int ho = (h - 1) / 2 + 1, wo = (w - 1) / 2 + 1;
    const long long total = static_cast<long long>(n) * ho * wo * 9 * (C / 8);
    im2col_s2_kernel<<<grid_for(total, 256), 256, 0, s>>>(static_cast<const uint16_t*>(x), n, h, w, C,
                                                          static_cast<uint16_t*>(out));
    M3R_CUDA(cudaGetLastError());
}

void retrieval_attention(cudaStream_t s, const float* w, int n_img, int N, int D, float* attn) {
    if (n_img <= 0) return;
    retrieval_attention_kernel<<<n_img, 512, 0, s>>>(w, N, D, attn);
    M3R_CUDA(cudaGetLastError());
}

void resize_crop(cudaStream_t s, const uint8_t* src, int sh, int sw, uint8_t* dst, int dh, int dw) {
    M3R_REQUIRE(sh > 0 && sw > 0 && dh > 0 && dw > 0, "resize_crop: bad size");
    // host side of preprocessing.cpp:34-41 (float arithmetic, as the reference)
    const float sc_h = static_cast<float>(dh) / static_cast<float>(sh);
    const float sc_w = static_cast<float>(dw) / static_cast<float>(sw);
    const float scale = sc_h > sc_w ? sc_h : sc_w;
    const int new_h = static_cast<int>(static_cast<float>(sh) * scale);
    const int new_w = static_cast<int>(static_cast<float>(sw) * scale);
    M3R_REQUIRE(new_h > 0 && new_w > 0, "resize_crop: degenerate resize");
    const float scale_y = static_cast<float>(sh) / static_cast<float>(new_h);
    const float scale_x = static_cast<float>(sw) / static_cast<float>(new_w);
    const long long total = static_cast<long long>(dh) * dw;
    resize_crop_kernel<<<grid_for(total, 256), 256, 0, s>>>(src, sh, sw, dst, dh, dw, new_h, new_w, scale_y, scale_x);
    M3R_CUDA(cudaGetLastError());
}

void upsample_ref(cudaStream_t s, const float* x, int n, int hi, int wi, int C, int ho, int wo, float* y) {
    M3R_REQUIRE(C % 4 == 0, "upsample_ref: channels must be a multiple of 4");
    M3R_REQUIRE(((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0,
                "upsample_ref: buffers must be 16-byte aligned");
    const long long total = static_cast<long long>(n) * ho * wo * (C / 4);
    upsample_ref_kernel<<<grid_for(total, 256), 256, 0, s>>>(reinterpret_cast<const float4*>(x), n, hi, wi, C / 4, ho,
                                                              wo, reinterpret_cast<float4*>(y));
    M3R_CUDA(cudaGetLastError());
}

void upsample_ref_split(cudaStream_t s, const float* x4, int n, int hi, int wi, int ho, int wo, float* pts3d,
                        float* conf) {
    const long long total = static_cast<long long>(n) * ho * wo;
    upsample_ref_split_kernel<<<grid_for(total, 256), 256, 0, s>>>(reinterpret_cast<const float4*>(x4), n, hi, wi, ho,
                                                                    wo, pts3d, conf);
    M3R_CUDA(cudaGetLastError());
}

void head_split(cudaStream_t s, const float* out4, int n, int h4, int w4, int H, int W, float* pts3d, float* conf) {
    const long long total = static_cast<long long>(n) * H * W;
    head_split_kernel<<<grid_for(total, 256), 256, 0, s>>>(out4, n, h4, w4, H, W, pts3d, conf);
    M3R_CUDA(cudaGetLastError());
}

}  // namespace m3r
