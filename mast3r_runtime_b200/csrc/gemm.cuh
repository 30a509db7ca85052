// Persistent tcgen05 GEMM for sm_100a:  C[M, N] = A[M, K] * B[N, K]^T  (fp16 or
// bf16 operands, fp32 accumulate in TMEM), with the fused epilogues of the
// two-view model.  T is the 16-bit operand type; 16-bit outputs are written as T.
//
// Roles (320 threads):  warps 0-7 epilogue, warp 8 TMA producer, warp 9 TMEM
// allocator + single-thread MMA issuer.  Epilogue warp w reads TMEM lanes
// 32*(w%4) .. +32 (= tile rows) and the column units of group w/4, so two warps
// share every TMEM lane quarter and split the tile's columns.
// Tiles are 128 x BN, K in blocks of 64 (one 128-byte swizzle atom per row); the
// accumulator is double-buffered in TMEM so that the epilogue of one tile
// overlaps the main loop of the next.  Tiles are visited N-fastest so that the
// 128-row A block is reused from L2 across the N tiles.
//
// A operand modes:
//   A_PLAIN   2-D tensor map [M, K]
//   A_CONCAT  two 2-D maps, K = K0 + K1 (the local-feature MLP input enc || dec)
//   A_CONV3   4-D map [img, H, W, C]: implicit-GEMM 3x3 convolution, stride 1,
//             pad 1; the 9 taps are TMA boxes shifted by (dy, dx), zero padding
//             comes from TMA out-of-bounds fill.  A tile is wbox x hbox pixels.
// Epilogues: see enum Epi.
#pragma once

#include "common.cuh"

namespace m3r {

enum AMode : int { A_PLAIN = 0, A_CONCAT = 1, A_CONV3 = 2 };

enum Epi : int {
    EPI_BF16 = 0,       // out_T = act(acc + bias)   (16-bit output of the operand type T)
    EPI_F32 = 1,        // out_f32 = acc + bias
    EPI_F32_RESID = 2,  // out_f32 = resid_f32 + acc + bias   (resid may alias out)
    EPI_HEADS = 3,      // + bias, optional 2-D RoPE, scatter to head-major [seq, head, tok, 64] T
    EPI_DESC = 4,       // + bias, pixel shuffle, L2-normalise groups of 24 -> fp32 descriptors
    EPI_HEAD4 = 5,      // + bias, ReLU, fused 1x1 conv 128 -> 4 (+ bias4) -> fp32 [pixel, 4]
    EPI_CONVT = 6,      // + bias, transposed conv (kernel == stride) scatter -> T NHWC
};

enum Act : int { ACT_NONE = 0, ACT_GELU = 1, ACT_RELU = 2 };

struct GemmParams {
    int M, N;          // output rows (plain/concat) and columns
    int num_kb;        // k-blocks (of 64) per tile
    int tiles_m, tiles_n;
    int a_split_kb;    // A_CONCAT: k-blocks taken from map A0
    // A_CONV3 geometry
    int cv_H, cv_W, cv_cblocks, cv_wbox, cv_hbox, cv_tx, cv_ty;
    // epilogue
    const float* bias;
    int act;
    void* out;
    long long ldo;     // elements
    const float* resid;
    long long ldr;
    // EPI_HEADS
    int sec_len, n_tok, grid_w;
    void* sec_out[3];
    int sec_rope[3];
    const float* rope_cos;  // [pos][16]
    const float* rope_sin;
    // EPI_DESC
    int patch, grid_h, desc_dim;
    // EPI_HEAD4
    const float* w4;   // [4][128]
    const float* b4;   // [4]
    // EPI_CONVT
    int ct_s, ct_cout, ct_h, ct_w;
    // device status word: a wait that runs out of time records its code here
    int* err;
};

constexpr int kGemmEpiWarps = 8;
constexpr int kGemmThreads = (kGemmEpiWarps + 2) * 32;
constexpr int kGemmTmaWarp = kGemmEpiWarps;
constexpr int kGemmMmaWarp = kGemmEpiWarps + 1;

template <int BN>
struct GemmCfg {
    static constexpr int BM = 128;
    static constexpr int BK = 64;
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES = (200 * 1024 / STAGE_BYTES) > 8 ? 8 : (200 * 1024 / STAGE_BYTES);
    static constexpr int ACC_COLS = BN <= 128 ? 128 : 256;   // per accumulator buffer
    static constexpr int TMEM_COLS = 2 * ACC_COLS;
    // stages | barriers, TMEM slot, abort flag (256 B) | EPI_HEAD4 partial sums [128][4] fp32
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 + 128 * 4 * 4;
};

struct TileGeom {
    int m_idx, n_idx;
    int img, y0, x0;  // A_CONV3 only
};

template <int AMODE>
__device__ __forceinline__ TileGeom tile_geom(const GemmParams& p, int t) {
    TileGeom g;
    g.m_idx = t / p.tiles_n;
    g.n_idx = t - g.m_idx * p.tiles_n;
    g.img = g.y0 = g.x0 = 0;
    if (AMODE == A_CONV3) {
        const int per_img = p.cv_tx * p.cv_ty;
        g.img = g.m_idx / per_img;
        const int rem = g.m_idx - g.img * per_img;
        const int ty = rem / p.cv_tx;
        g.y0 = ty * p.cv_hbox;
        g.x0 = (rem - ty * p.cv_tx) * p.cv_wbox;
    }
    return g;
}

// ------------------------------------------------------------------------- epilogue helpers
// GELU, tanh form (backends/python/vit_encoder.py:18-20), with the hardware tanh
// approximation (tanh.approx.f32, relative error about 2^-11 -- below the fp16
// rounding of the value it produces).
__device__ __forceinline__ float gelu_fast(float x) {
    const float k0 = 0.7978845608028654f;  // sqrt(2 / pi)
    const float k1 = 0.044715f;
    float t;
    const float u = k0 * (x + k1 * x * x * x);
    asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(u));
    return 0.5f * x * (1.0f + t);
}

template <class T>
__device__ __forceinline__ void store16x32(T* dst, const float (&v)[32]) {
    uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint4 u;
        u.x = Elem<T>::pack(v[q * 8 + 0], v[q * 8 + 1]);
        u.y = Elem<T>::pack(v[q * 8 + 2], v[q * 8 + 3]);
        u.z = Elem<T>::pack(v[q * 8 + 4], v[q * 8 + 5]);
        u.w = Elem<T>::pack(v[q * 8 + 6], v[q * 8 + 7]);
        d[q] = u;
    }
}

// bias[col0 .. col0+32) added to v; `full` = the 32 columns exist (bias 16-byte aligned)
__device__ __forceinline__ void add_bias32(float (&v)[32], const float* bias, int col0, int N, bool full) {
    if (bias == nullptr) return;
    if (full) {
        const float4* b4 = reinterpret_cast<const float4*>(bias + col0);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float4 b = __ldg(b4 + q);
            v[4 * q] += b.x;
            v[4 * q + 1] += b.y;
            v[4 * q + 2] += b.z;
            v[4 * q + 3] += b.w;
        }
    } else {
        for (int i = 0; i < 32; ++i)
            if (col0 + i < N) v[i] += __ldg(bias + col0 + i);
    }
}

// Epilogue of one tile for one column group (grp 0 / 1) of the rows of this thread
// (tile row r).  All lanes of a warp execute every tcgen05.ld (they are .sync.aligned).
// EPI_HEAD4 hand-off between the two column groups: partial sums in smem, guarded by
// two mbarriers (h4[0] "partials written", h4[1] "partials consumed") with bounded waits.
struct Head4Sync {
    float* part;       // [128][4]
    uint64_t* full;    // count 128: group 1 arrives after writing
    uint64_t* empty;   // count 128: group 0 arrives after reading
    volatile int* abort_flag;
    uint32_t tile;     // this CTA's tile counter (phase parity)
};

template <class T, int BN, int AMODE, int EPI>
__device__ __forceinline__ void epilogue_tile(const GemmParams& p, const TileGeom& g, uint32_t tacc, int r, int grp,
                                              const Head4Sync& h4) {
    // tile row r -> global output row
    long long grow;
    bool valid;
    if (AMODE == A_CONV3) {
        const int y = g.y0 + r / p.cv_wbox;
        const int x = g.x0 + r % p.cv_wbox;
        valid = y < p.cv_H;
        grow = (static_cast<long long>(g.img) * p.cv_H + y) * p.cv_W + x;
    } else {
        grow = static_cast<long long>(g.m_idx) * 128 + r;
        valid = grow < p.M;
    }
    const int n0 = g.n_idx * BN;

    if constexpr (EPI == EPI_BF16 || EPI == EPI_F32 || EPI == EPI_F32_RESID || EPI == EPI_CONVT) {
#pragma unroll 1
        for (int c0 = grp * 32; c0 < BN; c0 += 64) {
            const int col0 = n0 + c0;
            const bool full = col0 + 32 <= p.N;
            float v[32];
            // residual rows do not depend on the accumulator: fetch them before the TMEM read
            if constexpr (EPI == EPI_F32_RESID) {
                if (valid && full) {
                    const float4* src = reinterpret_cast<const float4*>(p.resid + grow * p.ldr + col0);
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const float4 rr = src[q];
                        v[4 * q] = rr.x;
                        v[4 * q + 1] = rr.y;
                        v[4 * q + 2] = rr.z;
                        v[4 * q + 3] = rr.w;
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = 0.0f;
                    if (valid)
                        for (int i = 0; i < 32 && col0 + i < p.N; ++i) v[i] = p.resid[grow * p.ldr + col0 + i];
                }
            }
            uint32_t raw[32];
            tmem_ld32(tacc + c0, raw);
            tmem_wait_ld();
            if (!valid || col0 >= p.N) continue;
            if constexpr (EPI == EPI_F32_RESID) {
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] += __uint_as_float(raw[i]);
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(raw[i]);
            }
            if constexpr (EPI == EPI_CONVT) {
                // column = (dy * s + dx) * cout + co, cout % 32 == 0: one bias window
                const int q = col0 / p.ct_cout;
                const int co = col0 - q * p.ct_cout;
                add_bias32(v, p.bias, co, p.ct_cout, true);
                const int dy = q / p.ct_s, dx = q - (q / p.ct_s) * p.ct_s;
                const int per_img = p.ct_h * p.ct_w;
                const int img = static_cast<int>(grow / per_img);
                const int rem = static_cast<int>(grow - static_cast<long long>(img) * per_img);
                const int yy = rem / p.ct_w, xx = rem - (rem / p.ct_w) * p.ct_w;
                const int OH = p.ct_h * p.ct_s, OW = p.ct_w * p.ct_s;
                const long long opix = (static_cast<long long>(img) * OH + (yy * p.ct_s + dy)) * OW + (xx * p.ct_s + dx);
                store16x32<T>(reinterpret_cast<T*>(p.out) + opix * p.ldo + co, v);
            } else {
                add_bias32(v, p.bias, col0, p.N, full);
                if constexpr (EPI == EPI_BF16) {
                    if (p.act == ACT_GELU) {
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = gelu_fast(v[i]);
                    } else if (p.act == ACT_RELU) {
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = fmaxf(v[i], 0.0f);
                    }
                    T* dst = reinterpret_cast<T*>(p.out) + grow * p.ldo + col0;
                    if (full) {
                        store16x32<T>(dst, v);
                    } else {
                        for (int i = 0; i < 32 && col0 + i < p.N; ++i) dst[i] = Elem<T>::from(v[i]);
                    }
                } else {
                    float* dst = reinterpret_cast<float*>(p.out) + grow * p.ldo + col0;
                    if (full) {
#pragma unroll
                        for (int q = 0; q < 8; ++q)
                            *reinterpret_cast<float4*>(dst + 4 * q) = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
                    } else {
                        for (int i = 0; i < 32 && col0 + i < p.N; ++i) dst[i] = v[i];
                    }
                }
            }
        }
    } else if constexpr (EPI == EPI_HEADS) {
        // The tile lies inside one section (sec_len % BN == 0); 64 columns = one head.
        const int sec = n0 / p.sec_len;
        const int nh = p.sec_len / 64;
        const int seq = static_cast<int>(grow / p.n_tok);
        const int tok = static_cast<int>(grow - static_cast<long long>(seq) * p.n_tok);
        const int py = tok / p.grid_w, px = tok - (tok / p.grid_w) * p.grid_w;
        const bool rope = p.sec_rope[sec] != 0;
        T* base = reinterpret_cast<T*>(p.sec_out[sec]);
#pragma unroll 1
        for (int c0 = grp * 64; c0 < BN; c0 += 128) {
            uint32_t ra[32], rb[32];
            tmem_ld32(tacc + c0, ra);
            tmem_ld32(tacc + c0 + 32, rb);
            tmem_wait_ld();
            if (!valid) continue;
            const int col0 = n0 + c0;
            const int head = (col0 - sec * p.sec_len) >> 6;
            float lo[32], hi[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                lo[i] = __uint_as_float(ra[i]);
                hi[i] = __uint_as_float(rb[i]);
            }
            add_bias32(lo, p.bias, col0, p.N, true);
            add_bias32(hi, p.bias, col0 + 32, p.N, true);
            if (rope) {
                // rope2d.py:133-146: pairs (i, i+32); i < 16 rotate by y*f_i, i >= 16 by x*f_(i-16)
                const float4* cy = reinterpret_cast<const float4*>(p.rope_cos + py * 16);
                const float4* sy = reinterpret_cast<const float4*>(p.rope_sin + py * 16);
                const float4* cx = reinterpret_cast<const float4*>(p.rope_cos + px * 16);
                const float4* sx = reinterpret_cast<const float4*>(p.rope_sin + px * 16);
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const float4 c4 = __ldg(q < 4 ? cy + q : cx + (q - 4));
                    const float4 s4 = __ldg(q < 4 ? sy + q : sx + (q - 4));
                    const float cc[4] = {c4.x, c4.y, c4.z, c4.w};
                    const float ss[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int i = 4 * q + e;
                        const float t1 = lo[i], t2 = hi[i];
                        lo[i] = t1 * cc[e] - t2 * ss[e];
                        hi[i] = t1 * ss[e] + t2 * cc[e];
                    }
                }
            }
            T* dst = base + ((static_cast<long long>(seq) * nh + head) * p.n_tok + tok) * 64;
            store16x32<T>(dst, lo);
            store16x32<T>(dst + 32, hi);
        }
    } else if constexpr (EPI == EPI_DESC) {
        // Columns are groups of 24 channels, one group per (dy, dx) of the patch
        // (pixel-shuffle order (dy, dx, c), mpsgraph_engine.mm:425-437).
        const int img = static_cast<int>(grow / p.n_tok);
        const int tok = static_cast<int>(grow - static_cast<long long>(img) * p.n_tok);
        const int gy = tok / p.grid_w, gx = tok - (tok / p.grid_w) * p.grid_w;
        const int OH = p.grid_h * p.patch, OW = p.grid_w * p.patch;
#pragma unroll 1
        for (int c0 = grp * 96; c0 < BN; c0 += 192) {
            uint32_t r0[32], r1[32], r2[32];
            tmem_ld32(tacc + c0, r0);
            tmem_ld32(tacc + c0 + 32, r1);
            tmem_ld32(tacc + c0 + 64, r2);
            tmem_wait_ld();
            if (!valid || n0 + c0 >= p.N) continue;
            float v[96];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                v[i] = __uint_as_float(r0[i]);
                v[32 + i] = __uint_as_float(r1[i]);
                v[64 + i] = __uint_as_float(r2[i]);
            }
            const float4* b4 = reinterpret_cast<const float4*>(p.bias + n0 + c0);
#pragma unroll
            for (int q = 0; q < 24; ++q) {
                const float4 b = __ldg(b4 + q);
                v[4 * q] += b.x;
                v[4 * q + 1] += b.y;
                v[4 * q + 2] += b.z;
                v[4 * q + 3] += b.w;
            }
#pragma unroll
            for (int gq = 0; gq < 4; ++gq) {
                const int gidx = (n0 + c0) / 24 + gq;
                const int dy = gidx / p.patch, dx = gidx - (gidx / p.patch) * p.patch;
                float ss = 0.0f;
#pragma unroll
                for (int c = 0; c < 24; ++c) ss += v[gq * 24 + c] * v[gq * 24 + c];
                const float inv = 1.0f / sqrtf(ss + 1e-8f);
                const long long opix = (static_cast<long long>(img) * OH + gy * p.patch + dy) * OW + gx * p.patch + dx;
                float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + opix * 24);
#pragma unroll
                for (int q = 0; q < 6; ++q)
                    dst[q] = make_float4(v[gq * 24 + 4 * q] * inv, v[gq * 24 + 4 * q + 1] * inv,
                                         v[gq * 24 + 4 * q + 2] * inv, v[gq * 24 + 4 * q + 3] * inv);
            }
        }
    } else if constexpr (EPI == EPI_HEAD4) {
        // BN == 128 == all channels of one pixel: relu(conv3x3 + b) then 1x1 conv to 4.
        // Group g takes columns [64 g, 64 g + 64); group 1 hands its partial sums to group 0.
        float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
#pragma unroll 1
        for (int c0 = grp * 64; c0 < grp * 64 + 64; c0 += 32) {
            uint32_t raw[32];
            tmem_ld32(tacc + c0, raw);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const int c = c0 + i;
                const float v = fmaxf(__uint_as_float(raw[i]) + __ldg(p.bias + c), 0.0f);
                o0 += v * __ldg(p.w4 + c);
                o1 += v * __ldg(p.w4 + 128 + c);
                o2 += v * __ldg(p.w4 + 256 + c);
                o3 += v * __ldg(p.w4 + 384 + c);
            }
        }
        const uint32_t ph = h4.tile & 1;
        if (grp == 1) {
            if (mbar_wait(h4.empty, ph ^ 1, h4.abort_flag, kDevTimeoutEpilogue, p.err)) {
                *reinterpret_cast<float4*>(h4.part + 4 * r) = make_float4(o0, o1, o2, o3);
                mbar_arrive(h4.full);
            }
        } else if (mbar_wait(h4.full, ph, h4.abort_flag, kDevTimeoutEpilogue, p.err)) {
            const float4 q = *reinterpret_cast<const float4*>(h4.part + 4 * r);
            mbar_arrive(h4.empty);
            if (valid) {
                float4* dst = reinterpret_cast<float4*>(p.out) + grow;
                *dst = make_float4(o0 + q.x + __ldg(p.b4), o1 + q.y + __ldg(p.b4 + 1), o2 + q.z + __ldg(p.b4 + 2),
                                   o3 + q.w + __ldg(p.b4 + 3));
            }
        }
    }
}

// ------------------------------------------------------------------------- kernel
template <class T, int BN, int AMODE, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap mapA0, const __grid_constant__ CUtensorMap mapA1,
                   const __grid_constant__ CUtensorMap mapB, const __grid_constant__ GemmParams p) {
    using C = GemmCfg<BN>;
    constexpr int STAGES = C::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * C::A_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES);
    uint64_t* full = bars;
    uint64_t* empty = bars + STAGES;
    uint64_t* tfull = bars + 2 * STAGES;
    uint64_t* tempty = bars + 2 * STAGES + 2;
    uint64_t* mma_done = bars + 2 * STAGES + 4;
    uint64_t* h4_full = bars + 2 * STAGES + 5;
    uint64_t* h4_empty = bars + 2 * STAGES + 6;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 7);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float* head4_part = reinterpret_cast<float*>(smem + STAGES * C::STAGE_BYTES + 256);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int num_tiles = p.tiles_m * p.tiles_n;

    if (warp == kGemmTmaWarp && lane == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], kGemmEpiWarps * 32);
        }
        mbar_init(mma_done, 1);
        mbar_init(h4_full, 128);
        mbar_init(h4_empty, 128);
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tmap(&mapA0);
        if (AMODE == A_CONCAT) prefetch_tmap(&mapA1);
        prefetch_tmap(&mapB);
    }
    if (warp == kGemmMmaWarp) tmem_alloc(tmem_slot, C::TMEM_COLS);
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == kGemmTmaWarp) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                const TileGeom g = tile_geom<AMODE>(p, t);
                for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
                    const int s = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1;
                    if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, kDevTimeoutProducer, p.err)) { ok = false; break; }
                    mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
                    uint8_t* a_dst = sA + s * C::A_BYTES;
                    if (AMODE == A_PLAIN) {
                        tma_load_2d(a_dst, &mapA0, &full[s], kb * 64, g.m_idx * 128);
                    } else if (AMODE == A_CONCAT) {
                        if (kb < p.a_split_kb)
                            tma_load_2d(a_dst, &mapA0, &full[s], kb * 64, g.m_idx * 128);
                        else
                            tma_load_2d(a_dst, &mapA1, &full[s], (kb - p.a_split_kb) * 64, g.m_idx * 128);
                    } else {
                        const int tap = kb / p.cv_cblocks;
                        const int cb = kb - tap * p.cv_cblocks;
                        const int dy = tap / 3 - 1, dx = tap % 3 - 1;
                        tma_load_4d(a_dst, &mapA0, &full[s], cb * 64, g.x0 + dx, g.y0 + dy, g.img);
                    }
                    tma_load_2d(sB + s * C::B_BYTES, &mapB, &full[s], kb * 64, g.n_idx * BN);
                }
            }
            if (!ok) {
                // drain: wait (bounded) for loads that may still be in flight
                const uint32_t first = it > STAGES ? it - STAGES : 0;
                for (uint32_t j = first; j < it; ++j) {
                    volatile int dummy = 0;
                    mbar_wait(&full[j % STAGES], (j / STAGES) & 1, &dummy, kDevTimeoutProducer, p.err);
                }
            }
        }
    } else if (warp == kGemmMmaWarp) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16kind<T>(128, BN, false, false);
            uint32_t it = 0, tcount = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++tcount) {
                const uint32_t buf = tcount & 1;
                const uint32_t tph = (tcount >> 1) & 1;
                if (!mbar_wait(&tempty[buf], tph ^ 1, abort_flag, kDevTimeoutMma, p.err)) { ok = false; break; }
                tc_fence_after();
                const uint32_t dacc = tmem_base + buf * C::ACC_COLS;
                for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
                    const int s = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1;
                    if (!mbar_wait(&full[s], ph, abort_flag, kDevTimeoutMma, p.err)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sA + s * C::A_BYTES);
                    const uint32_t b_addr = smem_u32(sB + s * C::B_BYTES);
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const uint64_t ad = umma_desc_sw128(a_addr + k * 32, 16, 1024);
                        const uint64_t bd = umma_desc_sw128(b_addr + k * 32, 16, 1024);
                        mma_f16_ss(dacc, ad, bd, idesc, (kb > 0 || k > 0) ? 1u : 0u);
                    }
                    mma_commit(&empty[s]);
                }
                if (ok) mma_commit(&tfull[buf]);
            }
            // all issued MMAs complete before the CTA may release TMEM
            mma_commit(mma_done);
            volatile int dummy = 0;
            mbar_wait(mma_done, 0, &dummy, kDevTimeoutMma, p.err);
        }
    } else {
        // ------------------------------------------------ epilogue (warps 0-7)
        const int quarter = warp & 3;
        const int grp = warp >> 2;
        const int r = quarter * 32 + lane;
        uint32_t tcount = 0;
        for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++tcount) {
            const uint32_t buf = tcount & 1;
            const uint32_t tph = (tcount >> 1) & 1;
            if (!mbar_wait(&tfull[buf], tph, abort_flag, kDevTimeoutEpilogue, p.err)) break;
            tc_fence_after();
            const TileGeom g = tile_geom<AMODE>(p, t);
            const uint32_t tacc = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * C::ACC_COLS;
            const Head4Sync h4{head4_part, h4_full, h4_empty, abort_flag, tcount};
            epilogue_tile<T, BN, AMODE, EPI>(p, g, tacc, r, grp, h4);
            tc_fence_before();
            mbar_arrive(&tempty[buf]);
        }
    }
    __syncthreads();
    if (warp == kGemmMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::TMEM_COLS);
    }
}

}  // namespace m3r
