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
//   A_CONV3W  the same convolution for tiles of 128 pixels of one image row (W a
//             multiple of 128): one 136-pixel box per (dy, 64-channel block), from
//             x0 - 1, serves the three dx taps (MMA operand start 0, 1 or 2 rows
//             into it), a third of A_CONV3's operand traffic.  CTA pairs only.
// Epilogues: see enum Epi.
#pragma once

#include "common.cuh"

namespace m3r {

enum AMode : int { A_PLAIN = 0, A_CONCAT = 1, A_CONV3 = 2, A_CONV3W = 3 };

enum Epi : int {
    EPI_BF16 = 0,       // out_T = act(acc + bias)   (16-bit output of the operand type T)
    EPI_F32 = 1,        // out_f32 = acc + bias
    EPI_F32_RESID = 2,  // out_f32 = resid_f32 + acc + bias   (resid may alias out)
    EPI_HEADS = 3,      // + bias, optional 2-D RoPE, scatter to head-major [seq, head, tok, 64] T
    EPI_DESC = 4,       // + bias, pixel shuffle, L2-normalise groups of 24 -> fp32 descriptors
    EPI_HEAD4 = 5,      // + bias, ReLU, fused 1x1 conv 128 -> 4 (+ bias4) -> fp32 [pixel, 4]
    EPI_CONVT = 6,      // + bias, transposed conv (kernel == stride) scatter -> T NHWC
    EPI_F32_RESID_LK = 7,  // EPI_F32_RESID for long K, chosen by the launcher: fewer residual
                           // buffers, more operand stages
};

enum Act : int { ACT_NONE = 0, ACT_GELU = 1, ACT_RELU = 2 };

struct GemmParams {
    int M, N;          // output rows (plain/concat) and columns
    int num_kb;        // k-blocks (of 64) per tile; A_CONV3W: (dy, channel block) groups of 3 k-blocks
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
    const float* rope_cos;  // [16 frequencies][rope_npos positions]
    const float* rope_sin;
    int rope_npos;
    // EPI_DESC
    int patch, grid_h, desc_dim;
    // EPI_HEAD4
    const float* w4;   // [4][128]
    const float* b4;   // [4]
    // EPI_CONVT
    int ct_s, ct_cout, ct_h, ct_w;
    // 1: the output goes out through TMA stores of whole 32-row boxes (maps C0-C2:
    // the output matrix, or the three head-major sections of EPI_HEADS)
    int c_tma;
    // device status word: a wait that runs out of time records its code here
    int* err;
};

struct StoreMaps {
    const CUtensorMap* c[3];
};

constexpr int kGemmEpiWarps = 8;
constexpr int kGemmThreads = (kGemmEpiWarps + 2) * 32;
constexpr int kGemmTmaWarp = kGemmEpiWarps;
constexpr int kGemmMmaWarp = kGemmEpiWarps + 1;

// CG = CTAs per tile: 1, or 2 for a CTA pair (cluster of 2) running M = 256 MMAs,
// in which each CTA stages its own 128 rows of A and half of the tile's BN rows
// of B, and holds its 128 x BN accumulator rows in its own TMEM.
// A_CONV3W stages one 136-pixel A box and the B blocks of three taps per stage.
// Residual epilogues: 4 KB residual buffers per epilogue warp (a ring; see
// resid_epilogue), traded against operand stages.  Short K (the attention output
// projections, K <= 1024) is bound by the residual traffic: CTA pairs keep 3 buffers
// (4 operand stages at BN = 256).  Long K (the MLP outputs) is bound by the MMAs and
// keeps 2 (5 stages); so do single CTAs.
template <int EPI, int CG>
constexpr int epi_ring() {
    return EPI == EPI_F32_RESID ? (CG == 2 ? 3 : 2) : EPI == EPI_F32_RESID_LK ? 2 : 1;
}
template <int EPI>
constexpr bool epi_resid() {
    return EPI == EPI_F32_RESID || EPI == EPI_F32_RESID_LK;
}

template <int BN, int CG, int AMODE = A_PLAIN, int RING = 1>
struct GemmCfg {
    static constexpr int BM = 128;
    static constexpr int BK = 64;
    static constexpr int RING_BUFS = RING;
    static constexpr int B_ROWS = BN / CG;  // rows of B staged by each CTA
    static constexpr int WIDE_ROWS = 136;   // A_CONV3W box: 128 pixels + 2 halo, rounded to 8 rows
    static constexpr int TAPS = AMODE == A_CONV3W ? 3 : 1;  // B blocks per stage
    static constexpr int A_BYTES = (AMODE == A_CONV3W ? WIDE_ROWS : BM) * BK * 2;
    static constexpr int B_TAP_BYTES = B_ROWS * BK * 2;
    static constexpr int B_BYTES = TAPS * B_TAP_BYTES;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    // per-epilogue-warp row staging, RING x 4 KB each (EPI_HEAD4 keeps its partial sums there)
    static constexpr int EPI_STAGE_BYTES = kGemmEpiWarps * 4096 * RING;
    // stages | epilogue staging | barriers, TMEM slot, abort flag (256 B) | ring barriers;
    // + 1 KB alignment slack
    static constexpr int RING_BAR_BYTES = RING > 1 ? kGemmEpiWarps * RING * 8 : 0;
    static constexpr int FIXED_BYTES = 1024 + EPI_STAGE_BYTES + 256 + RING_BAR_BYTES;
    static constexpr int MAX_SMEM = 227 * 1024;  // per-block opt-in limit of sm_100
    static constexpr int STAGES =
        ((MAX_SMEM - FIXED_BYTES) / STAGE_BYTES) > 8 ? 8 : ((MAX_SMEM - FIXED_BYTES) / STAGE_BYTES);
    static constexpr int ACC_COLS = BN <= 128 ? 128 : 256;   // per accumulator buffer
    static constexpr int TMEM_COLS = 2 * ACC_COLS;
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + FIXED_BYTES;
    static_assert(STAGES >= 3 && SMEM_BYTES <= MAX_SMEM, "shared memory budget");
    static_assert(BN % (8 * CG) == 0 && B_TAP_BYTES % 1024 == 0 && A_BYTES % 1024 == 0,
                  "operand tiles must be whole swizzle atoms");
    static_assert(AMODE != A_CONV3W || CG == 2, "A_CONV3W runs on CTA pairs");
};

struct TileGeom {
    int m_idx, n_idx;
    bool live;        // the 128-row block exists (a CTA pair's odd block may lie past the last one)
    int img, y0, x0;  // A_CONV3 only
};

// Tile t of the persistent loop (N-fastest); a CTA pair covers row blocks 2 m + rank.
template <int AMODE, int CG>
__device__ __forceinline__ TileGeom tile_geom(const GemmParams& p, int t, int rank) {
    TileGeom g;
    const int mp = t / p.tiles_n;
    g.n_idx = t - mp * p.tiles_n;
    g.m_idx = mp * CG + rank;
    g.live = g.m_idx < p.tiles_m;
    g.img = g.y0 = g.x0 = 0;
    if (AMODE == A_CONV3 || AMODE == A_CONV3W) {
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

// 64 values (lo = columns 0-31, hi = 32-63) -> 128 bytes of the 16-bit type T
template <class T>
__device__ __forceinline__ void pack16x64(uint4 (&u)[8], const float (&lo)[32], const float (&hi)[32]) {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        const float* v = q < 4 ? lo + 8 * q : hi + 8 * (q - 4);
        u[q].x = Elem<T>::pack(v[0], v[1]);
        u[q].y = Elem<T>::pack(v[2], v[3]);
        u[q].z = Elem<T>::pack(v[4], v[5]);
        u[q].w = Elem<T>::pack(v[6], v[7]);
    }
}

// Per-warp staging of a 32-row x 128-byte block in shared memory, so that global
// memory sees whole 128-byte lines.  Each thread owns one row (its TMEM lane); the
// 16-byte chunks of row r sit at chunk position c ^ (r % 8), which makes both
// row-per-thread accesses and row-contiguous accesses (8 threads per row, 4 rows
// per instruction) free of bank conflicts.
struct RowStage {
    uint8_t* buf;  // 4 KB of this warp
    int lane;
    __device__ __forceinline__ uint4* at(int row, int c) const {
        return reinterpret_cast<uint4*>(buf + row * 128 + ((c ^ (row & 7)) << 4));
    }
    __device__ __forceinline__ void put_own(const uint4 (&v)[8]) const {
#pragma unroll
        for (int c = 0; c < 8; ++c) *at(lane, c) = v[c];
    }
    __device__ __forceinline__ void get_own(uint4 (&v)[8]) const {
#pragma unroll
        for (int c = 0; c < 8; ++c) v[c] = *at(lane, c);
    }
    // Row-contiguous global stores of the staged rows (dst = each thread's own row
    // pointer, null = skip; `bytes` = valid bytes per row, a multiple of 2).
    __device__ __forceinline__ void store(char* dst, int bytes) const {
        const int c = lane & 7;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int row = i * 4 + (lane >> 3);
            char* d = reinterpret_cast<char*>(__shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(dst), row));
            const uint4 v = *at(row, c);
            if (d != nullptr) {
                if ((c + 1) * 16 <= bytes) {
                    *reinterpret_cast<uint4*>(d + c * 16) = v;
                } else if (c * 16 < bytes) {
                    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
                    for (int b = 0; b < 8 && c * 16 + 2 * b < bytes; ++b)
                        *reinterpret_cast<uint16_t*>(d + c * 16 + 2 * b) =
                            static_cast<uint16_t>(w[b >> 1] >> ((b & 1) * 16));
                }
            }
        }
    }
};

// Epilogue of one tile for one column group (grp 0 / 1) of the rows of this thread
// (tile row r).  All lanes of a warp execute every tcgen05.ld (they are .sync.aligned).
// EPI_HEAD4 hand-off between the two column groups: partial sums in smem, guarded by
// two mbarriers (h4[0] "partials written", h4[1] "partials consumed") with bounded waits.
struct Head4Sync {
    float* part;       // [128][4]
    const float* wts;  // [128] float4 1x1 weights (channel-major) + [128] bias, in shared memory
    uint64_t* full;    // count 128: group 1 arrives after writing
    uint64_t* empty;   // count 128: group 0 arrives after reading
    volatile int* abort_flag;
    uint32_t tile;     // this CTA's tile counter (phase parity)
};

// Tile row r -> global output row (grow) and whether it exists.
template <int AMODE>
__device__ __forceinline__ void tile_row(const GemmParams& p, const TileGeom& g, int r, long long& grow, bool& valid) {
    if (AMODE == A_CONV3 || AMODE == A_CONV3W) {
        const int y = g.y0 + r / p.cv_wbox;
        const int x = g.x0 + r % p.cv_wbox;
        valid = y < p.cv_H;
        grow = (static_cast<long long>(g.img) * p.cv_H + y) * p.cv_W + x;
    } else {
        grow = static_cast<long long>(g.m_idx) * 128 + r;
        valid = grow < p.M;
    }
}

template <class T, int BN, int AMODE, int EPI>
__device__ __forceinline__ void epilogue_tile(const GemmParams& p, const TileGeom& g, uint32_t tacc, int r, int grp,
                                              const Head4Sync& h4, const RowStage& st, const StoreMaps& maps) {
    long long grow;
    bool valid;
    tile_row<AMODE>(p, g, r, grow, valid);
    const int n0 = g.n_idx * BN;
    // TMA stores: the warp's 32 rows are consecutive output rows starting at wrow0
    // (A_CONV3 only with boxes at least 32 pixels wide); wok = that row exists
    long long wrow0;
    bool wok;
    tile_row<AMODE>(p, g, r - st.lane, wrow0, wok);
    const int lane = st.lane;

    if constexpr (EPI == EPI_F32) {
        // units of 32 fp32 columns = 128 bytes per row, staged and stored row-contiguously
#pragma unroll 1
        for (int c0 = grp * 32; c0 < BN; c0 += 64) {
            const int col0 = n0 + c0;
            if (col0 >= p.N) break;  // warp-uniform
            const bool full = col0 + 32 <= p.N;
            uint32_t raw[32];
            tmem_ld32(tacc + c0, raw);
            tmem_wait_ld();
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(raw[i]);
            if (p.c_tma && lane == 0) bulk_wait_read_all();
            __syncwarp();  // the previous unit's reads of the stage (threads or TMA) are done
            add_bias32(v, p.bias, col0, p.N, full);
            uint4 o[8];
#pragma unroll
            for (int q = 0; q < 8; ++q)
                o[q] = make_uint4(__float_as_uint(v[4 * q]), __float_as_uint(v[4 * q + 1]), __float_as_uint(v[4 * q + 2]),
                                  __float_as_uint(v[4 * q + 3]));
            st.put_own(o);
            if (p.c_tma) {
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0 && wok) {
                    tma_store_2d(maps.c[0], st.buf, col0, static_cast<int>(wrow0));
                    bulk_commit();
                }
            } else {
                __syncwarp();
                st.store(valid ? reinterpret_cast<char*>(reinterpret_cast<float*>(p.out) + grow * p.ldo + col0)
                               : nullptr,
                         (full ? 32 : p.N - col0) * 4);
            }
        }
    } else if constexpr (EPI == EPI_BF16) {
        // units of 64 16-bit columns = 128 bytes per row, staged and stored row-contiguously
#pragma unroll 1
        for (int c0 = grp * 64; c0 < BN; c0 += 128) {
            const int col0 = n0 + c0;
            if (col0 >= p.N) break;  // warp-uniform
            uint32_t ra[32], rb[32];
            tmem_ld32(tacc + c0, ra);
            tmem_ld32(tacc + c0 + 32, rb);
            tmem_wait_ld();
            float lo[32], hi[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                lo[i] = __uint_as_float(ra[i]);
                hi[i] = __uint_as_float(rb[i]);
            }
            add_bias32(lo, p.bias, col0, p.N, col0 + 32 <= p.N);
            add_bias32(hi, p.bias, col0 + 32, p.N, col0 + 64 <= p.N);
            if (p.act == ACT_GELU) {
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    lo[i] = gelu_fast(lo[i]);
                    hi[i] = gelu_fast(hi[i]);
                }
            } else if (p.act == ACT_RELU) {
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    lo[i] = fmaxf(lo[i], 0.0f);
                    hi[i] = fmaxf(hi[i], 0.0f);
                }
            }
            uint4 o[8];
            pack16x64<T>(o, lo, hi);
            if (p.c_tma && lane == 0) bulk_wait_read_all();
            __syncwarp();
            st.put_own(o);
            if (p.c_tma) {
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0 && wok) {
                    tma_store_2d(maps.c[0], st.buf, col0, static_cast<int>(wrow0));
                    bulk_commit();
                }
            } else {
                __syncwarp();
                st.store(valid ? reinterpret_cast<char*>(reinterpret_cast<T*>(p.out) + grow * p.ldo + col0) : nullptr,
                         (col0 + 64 <= p.N ? 64 : p.N - col0) * 2);
            }
        }
    } else if constexpr (EPI == EPI_CONVT) {
#pragma unroll 1
        for (int c0 = grp * 32; c0 < BN; c0 += 64) {
            const int col0 = n0 + c0;
            uint32_t raw[32];
            tmem_ld32(tacc + c0, raw);
            tmem_wait_ld();
            if (!valid || col0 >= p.N) continue;
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(raw[i]);
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
        }
    } else if constexpr (EPI == EPI_HEADS) {
        // The tile lies inside one section (sec_len % BN == 0); 64 columns = one head,
        // 128 bytes per row of the head-major output, staged and stored row-contiguously.
        const int sec = n0 / p.sec_len;
        const int nh = p.sec_len / 64;
        const long long vrow = valid ? grow : 0;  // absent rows: in-range table indices, no store
        const int seq = static_cast<int>(vrow / p.n_tok);
        const int tok = static_cast<int>(vrow - static_cast<long long>(seq) * p.n_tok);
        const int py = tok / p.grid_w, px = tok - (tok / p.grid_w) * p.grid_w;
        const bool rope = p.sec_rope[sec] != 0;
        T* base = reinterpret_cast<T*>(p.sec_out[sec]);
#pragma unroll 1
        for (int c0 = grp * 64; c0 < BN; c0 += 128) {
            uint32_t ra[32], rb[32];
            tmem_ld32(tacc + c0, ra);
            tmem_ld32(tacc + c0 + 32, rb);
            tmem_wait_ld();
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
                // rope2d.py:133-146: pairs (i, i+32); i < 16 rotate by y*f_i, i >= 16 by x*f_(i-16).
                // Tables are frequency-major [16][npos]: a warp's 32 rows are consecutive tokens,
                // so their x lookups are one contiguous line and their y lookups mostly one value.
                const float* ctab = p.rope_cos;
                const float* stab = p.rope_sin;
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const int at = (i & 15) * p.rope_npos + (i < 16 ? py : px);
                    const float cc = __ldg(ctab + at), ss = __ldg(stab + at);
                    const float t1 = lo[i], t2 = hi[i];
                    lo[i] = t1 * cc - t2 * ss;
                    hi[i] = t1 * ss + t2 * cc;
                }
            }
            uint4 o[8];
            pack16x64<T>(o, lo, hi);
            if (p.c_tma && lane == 0) bulk_wait_read_all();
            __syncwarp();
            st.put_own(o);
            if (p.c_tma) {
                // n_tok % 32 == 0: the warp's rows are tokens tok0 .. tok0 + 31 of one sequence
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0 && wok) {
                    const int seq0 = static_cast<int>(wrow0 / p.n_tok);
                    const int tok0 = static_cast<int>(wrow0 - static_cast<long long>(seq0) * p.n_tok);
                    tma_store_3d(maps.c[sec], st.buf, 0, tok0, seq0 * nh + head);
                    bulk_commit();
                }
            } else {
                __syncwarp();
                T* dst = base + ((static_cast<long long>(seq) * nh + head) * p.n_tok + tok) * 64;
                st.store(valid ? reinterpret_cast<char*>(dst) : nullptr, 128);
            }
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
        // The bias and the 1x1 weights (column-major, one float4 per channel) sit in
        // shared memory (Head4Sync::wts), read as warp-wide broadcasts.
        float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
        const float4* wt = reinterpret_cast<const float4*>(h4.wts);   // [128] (w0c, w1c, w2c, w3c)
        const float4* bs = reinterpret_cast<const float4*>(h4.wts + 4 * 128);  // bias, [32] float4
#pragma unroll 1
        for (int c0 = grp * 64; c0 < grp * 64 + 64; c0 += 32) {
            uint32_t raw[32];
            tmem_ld32(tacc + c0, raw);
            tmem_wait_ld();
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float4 b = bs[(c0 >> 2) + q];
                const float bb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float4 w = wt[c0 + 4 * q + e];
                    const float v = fmaxf(__uint_as_float(raw[4 * q + e]) + bb[e], 0.0f);
                    o0 += v * w.x;
                    o1 += v * w.y;
                    o2 += v * w.z;
                    o3 += v * w.w;
                }
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
// CG = 2: launched as clusters of 2 CTAs (grid = 2 x pairs).  The even CTA's
// thread issues the M = 256 MMAs; both CTAs run producer and epilogue roles on
// the same tile sequence.  A wait that runs out raises the abort flag of both
// CTAs; neither CTA leaves before the other (cluster barrier at the end).
// EPI_F32_RESID epilogue of one warp over all of its tiles: out = (acc + resid) + bias
// in fp32 (resid may alias out).  The warp's units are 32 rows x 32 columns (4 KB):
// columns grp * 32 + 64 j of each tile.  Each unit's residual block arrives by TMA in
// one of RING 4 KB buffers, each with its own mbarrier; lane 0 issues the load of unit
// u + RING - 1 once unit u has been stored, across tile boundaries (the residual does
// not depend on the accumulator), so RING - 1 blocks per warp stay in flight from HBM
// while the warp works.  The sum overwrites the residual in the same buffer (one row
// per thread; the 128-byte swizzle of the box keeps row-per-thread accesses free of
// bank conflicts) and leaves by TMA store.  The tile's TMEM buffer is released after
// its last tcgen05.ld.
template <int BN, int AMODE, int CG, int RING, class Abort>
__device__ __forceinline__ void resid_epilogue(const GemmParams& p, uint32_t tmem_base, uint64_t* tfull,
                                               uint64_t* tempty, uint32_t tempty_c, uint64_t* rbar, uint8_t* ring,
                                               const CUtensorMap* map_out, const CUtensorMap* map_resid,
                                               volatile int* abort_flag, Abort&& abort_pair, int quarter, int grp,
                                               int lane, int rank, int unit, int num_units, int num_tiles) {
    static_assert(AMODE == A_PLAIN && RING >= 2, "residual epilogue: plain A, at least two buffers");
    constexpr uint32_t kAccCols = BN <= 128 ? 128 : 256;
    // units of this warp in a tile (0 when its row block does not exist)
    auto tile_units = [&](const TileGeom& g) -> int {
        if (!g.live) return 0;
        const int lim = p.N - g.n_idx * BN < BN ? p.N - g.n_idx * BN : BN;
        return lim > grp * 32 ? (lim - grp * 32 + 63) / 64 : 0;
    };
    // load cursor (lane 0): tile lt, unit lj of it, lu units issued so far
    int lt = unit, lj = 0;
    uint32_t lu = 0;
    auto issue = [&]() {
        while (lt < num_tiles) {
            const TileGeom g = tile_geom<AMODE, CG>(p, lt, rank);
            if (lj < tile_units(g)) {
                const int b = static_cast<int>(lu % RING);
                const int row0 = g.m_idx * 128 + quarter * 32;
                if (row0 < p.M) {
                    mbar_arrive_expect_tx(&rbar[b], 4096);
                    tma_load_2d(ring + b * 4096, map_resid, &rbar[b], g.n_idx * BN + grp * 32 + 64 * lj, row0);
                } else {
                    mbar_arrive(&rbar[b]);  // rows past the end: nothing to load or store
                }
                ++lj;
                ++lu;
                return;
            }
            lt += num_units;
            lj = 0;
        }
    };
    if (lane == 0)
        for (int i = 0; i < RING - 1; ++i) issue();

    uint32_t cu = 0, tcount = 0;  // units consumed, tiles visited
    bool ok = true;
    for (int t = unit; t < num_tiles && ok; t += num_units, ++tcount) {
        const uint32_t buf = tcount & 1;
        const TileGeom g = tile_geom<AMODE, CG>(p, t, rank);
        if (!mbar_wait(&tfull[buf], (tcount >> 1) & 1, abort_flag, kDevTimeoutEpilogue, p.err)) {
            abort_pair();
            ok = false;
            break;
        }
        tc_fence_after();
        const int nu = tile_units(g);
        const int row0 = g.m_idx * 128 + quarter * 32;
        const bool rows_ok = row0 < p.M;
        const uint32_t tacc = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * kAccCols;
        auto release = [&]() {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (CG == 2)
                    mbar_arrive_cluster(tempty_c + buf * 8);
                else
                    mbar_arrive(&tempty[buf]);
            }
        };
        if (nu == 0) release();
#pragma unroll 1
        for (int j = 0; j < nu; ++j, ++cu) {
            const int c0 = grp * 32 + 64 * j;
            const int col0 = g.n_idx * BN + c0;
            uint32_t raw[32];
            tmem_ld32(tacc + c0, raw);
            tmem_wait_ld();
            if (j == nu - 1) release();
            const int b = static_cast<int>(cu % RING);
            if (!mbar_wait(&rbar[b], (cu / RING) & 1, abort_flag, kDevTimeoutEpilogue, p.err)) {
                abort_pair();
                ok = false;
                break;
            }
            const RowStage rs{ring + b * 4096, lane};
            uint4 rr[8];
            rs.get_own(rr);
            float v[32];
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                v[4 * q] = __uint_as_float(raw[4 * q]) + __uint_as_float(rr[q].x);
                v[4 * q + 1] = __uint_as_float(raw[4 * q + 1]) + __uint_as_float(rr[q].y);
                v[4 * q + 2] = __uint_as_float(raw[4 * q + 2]) + __uint_as_float(rr[q].z);
                v[4 * q + 3] = __uint_as_float(raw[4 * q + 3]) + __uint_as_float(rr[q].w);
            }
            add_bias32(v, p.bias, col0, p.N, col0 + 32 <= p.N);
            uint4 o[8];
#pragma unroll
            for (int q = 0; q < 8; ++q)
                o[q] = make_uint4(__float_as_uint(v[4 * q]), __float_as_uint(v[4 * q + 1]), __float_as_uint(v[4 * q + 2]),
                                  __float_as_uint(v[4 * q + 3]));
            rs.put_own(o);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                // the buffer refilled next, (cu + RING - 1) % RING, was stored from by the
                // previous unit: its store must have finished reading it
                if (rows_ok) {
                    tma_store_2d(map_out, rs.buf, col0, row0);
                    bulk_commit();
                    bulk_wait_read_1();
                } else {
                    bulk_wait_read_all();
                }
                issue();
            }
        }
    }
    if (!ok && lane == 0) {
        // wait (bounded) for the residual loads still in flight before the CTA may leave
        volatile int no_abort = 0;
        for (uint32_t u = cu; u < lu; ++u)
            mbar_wait(&rbar[u % RING], (u / RING) & 1, &no_abort, kDevTimeoutEpilogue, p.err);
    }
}

template <class T, int BN, int AMODE, int EPI, int CG>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap mapA0, const __grid_constant__ CUtensorMap mapA1,
                   const __grid_constant__ CUtensorMap mapB, const __grid_constant__ CUtensorMap mapC0,
                   const __grid_constant__ CUtensorMap mapC1, const __grid_constant__ CUtensorMap mapC2,
                   const __grid_constant__ GemmParams p) {
    static_assert(CG == 1 || CG == 2, "one CTA or a CTA pair per tile");
    using C = GemmCfg<BN, CG, AMODE, epi_ring<EPI, CG>()>;
    constexpr int STAGES = C::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * C::A_BYTES;
    uint8_t* epi_stage = smem + STAGES * C::STAGE_BYTES;  // 1024-aligned: stage sizes are whole KB
    uint64_t* bars = reinterpret_cast<uint64_t*>(epi_stage + C::EPI_STAGE_BYTES);
    uint64_t* full = bars;
    uint64_t* empty = bars + STAGES;
    uint64_t* tfull = bars + 2 * STAGES;
    uint64_t* tempty = bars + 2 * STAGES + 2;
    uint64_t* mma_done = bars + 2 * STAGES + 4;
    uint64_t* h4_full = bars + 2 * STAGES + 5;
    uint64_t* h4_empty = bars + 2 * STAGES + 6;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 7);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    uint64_t* ring_bars = bars + 32;  // EPI_F32_RESID: RING per epilogue warp, after the 256-byte block
    float* head4_part = reinterpret_cast<float*>(epi_stage);
    float* head4_wts = reinterpret_cast<float*>(epi_stage + 2048);  // EPI_HEAD4: 640 floats

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int rank = CG == 2 ? static_cast<int>(cluster_rank()) : 0;
    const bool leader = rank == 0;
    const int unit = blockIdx.x / CG;        // CTA or CTA pair
    const int num_units = gridDim.x / CG;
    const int num_tiles = ((p.tiles_m + CG - 1) / CG) * p.tiles_n;

    if (warp == kGemmTmaWarp && lane == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], CG * kGemmEpiWarps);  // one arrival per epilogue warp of each CTA
        }
        mbar_init(mma_done, 1);
        mbar_init(h4_full, 128);
        mbar_init(h4_empty, 128);
        if (epi_resid<EPI>())
            for (int b = 0; b < kGemmEpiWarps * C::RING_BUFS; ++b) mbar_init(&ring_bars[b], 1);
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tmap(&mapA0);
        if (AMODE == A_CONCAT) prefetch_tmap(&mapA1);
        prefetch_tmap(&mapB);
    }
    if (EPI == EPI_HEAD4 && warp < kGemmEpiWarps) {
        // stage the 1x1 weights transposed (w[o][c] -> wts[4 c + o]) and the bias
        for (int i = threadIdx.x; i < 128; i += kGemmEpiWarps * 32) {
            head4_wts[4 * i + 0] = p.w4[i];
            head4_wts[4 * i + 1] = p.w4[128 + i];
            head4_wts[4 * i + 2] = p.w4[256 + i];
            head4_wts[4 * i + 3] = p.w4[384 + i];
            head4_wts[512 + i] = p.bias[i];
        }
    }
    if (warp == kGemmMmaWarp) {
        if (CG == 2)
            tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
        else
            tmem_alloc(tmem_slot, C::TMEM_COLS);
    }
    tc_fence_before();
    if (CG == 2)
        cluster_sync();  // barriers of both CTAs initialised before any cross-CTA signal
    else
        __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // shared::cluster addresses: the even CTA's full / tmem-empty barriers, the peer's abort flag
    const uint32_t full_c = CG == 2 ? cluster_addr(smem_u32(full), 0) : smem_u32(full);
    const uint32_t tempty_c = CG == 2 ? cluster_addr(smem_u32(tempty), 0) : smem_u32(tempty);
    const uint32_t peer_abort_c =
        CG == 2 ? cluster_addr(smem_u32(const_cast<int*>(abort_flag)), static_cast<uint32_t>(rank ^ 1)) : 0u;
    auto abort_pair = [&]() {
        *abort_flag = 1;
        if (CG == 2) st_cluster_u32(peer_abort_c, 1u);
    };

    if (warp == kGemmTmaWarp) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (int t = unit; t < num_tiles && ok; t += num_units) {
                const TileGeom g = tile_geom<AMODE, CG>(p, t, rank);
                for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
                    const int s = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1;
                    if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, kDevTimeoutProducer, p.err)) {
                        ok = false;
                        abort_pair();
                        break;
                    }
                    // the even CTA's full barrier counts the bytes of both CTAs
                    if (leader) mbar_arrive_expect_tx(&full[s], CG * C::STAGE_BYTES);
                    uint8_t* a_dst = sA + s * C::A_BYTES;
                    uint8_t* b_dst = sB + s * C::B_BYTES;
                    const uint32_t bar = full_c + s * 8;
                    const int brow = g.n_idx * BN + rank * C::B_ROWS;
                    if (CG == 2) {
                        if (AMODE == A_PLAIN) {
                            tma_load_2d_pair(a_dst, &mapA0, bar, kb * 64, g.m_idx * 128);
                        } else if (AMODE == A_CONCAT) {
                            if (kb < p.a_split_kb)
                                tma_load_2d_pair(a_dst, &mapA0, bar, kb * 64, g.m_idx * 128);
                            else
                                tma_load_2d_pair(a_dst, &mapA1, bar, (kb - p.a_split_kb) * 64, g.m_idx * 128);
                        } else if (AMODE == A_CONV3) {
                            const int tap = kb / p.cv_cblocks;
                            const int cb = kb - tap * p.cv_cblocks;
                            const int dy = tap / 3 - 1, dx = tap % 3 - 1;
                            tma_load_4d_pair(a_dst, &mapA0, bar, cb * 64, g.x0 + dx, g.y0 + dy, g.img);
                        } else {
                            // group kb = (dy, channel block): one wide A box, B of taps (dy, -1..1)
                            const int dyi = kb / p.cv_cblocks;
                            const int cb = kb - dyi * p.cv_cblocks;
                            tma_load_4d_pair(a_dst, &mapA0, bar, cb * 64, g.x0 - 1, g.y0 + dyi - 1, g.img);
                            for (int j = 0; j < 3; ++j)
                                tma_load_2d_pair(b_dst + j * C::B_TAP_BYTES, &mapB, bar,
                                                 ((dyi * 3 + j) * p.cv_cblocks + cb) * 64, brow);
                        }
                        if (AMODE != A_CONV3W) tma_load_2d_pair(b_dst, &mapB, bar, kb * 64, brow);
                    } else {
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
                        tma_load_2d(b_dst, &mapB, &full[s], kb * 64, brow);
                    }
                }
            }
            if (!ok) {
                if (CG == 1) {
                    // drain: wait (bounded) for loads that may still be in flight
                    const uint32_t first = it > STAGES ? it - STAGES : 0;
                    for (uint32_t j = first; j < it; ++j) {
                        volatile int dummy = 0;
                        mbar_wait(&full[j % STAGES], (j / STAGES) & 1, &dummy, kDevTimeoutProducer, p.err);
                    }
                } else {
                    // this CTA's loads signal the even CTA's barriers: give loads in flight
                    // 1 ms (TMA loads take microseconds) before the CTA may leave
                    const unsigned long long t0 = global_timer_ns();
                    while (global_timer_ns() - t0 < 1000000ull) __nanosleep(1000);
                }
            }
        }
    } else if (warp == kGemmMmaWarp) {
        // ------------------------------------------------ MMA issuer (even CTA of a pair)
        if (lane == 0 && leader) {
            constexpr uint32_t idesc = idesc_f16kind<T>(128 * CG, BN, false, false);
            uint32_t it = 0, tcount = 0;
            bool ok = true;
            for (int t = unit; t < num_tiles && ok; t += num_units, ++tcount) {
                const uint32_t buf = tcount & 1;
                const uint32_t tph = (tcount >> 1) & 1;
                if (!mbar_wait(&tempty[buf], tph ^ 1, abort_flag, kDevTimeoutMma, p.err)) {
                    ok = false;
                    abort_pair();
                    break;
                }
                tc_fence_after();
                const uint32_t dacc = tmem_base + buf * C::ACC_COLS;
                for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
                    const int s = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1;
                    if (!mbar_wait(&full[s], ph, abort_flag, kDevTimeoutMma, p.err)) {
                        ok = false;
                        abort_pair();
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sA + s * C::A_BYTES);
                    const uint32_t b_addr = smem_u32(sB + s * C::B_BYTES);
                    // A_CONV3W: tap dx = j - 1 reads the wide box from row j (pixel x0 + dx)
#pragma unroll
                    for (int j = 0; j < C::TAPS; ++j)
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const uint64_t ad = umma_desc_sw128(a_addr + j * 128 + k * 32, 16, 1024);
                            const uint64_t bd = umma_desc_sw128(b_addr + j * C::B_TAP_BYTES + k * 32, 16, 1024);
                            const uint32_t acc = (kb > 0 || j > 0 || k > 0) ? 1u : 0u;
                            if (CG == 2)
                                mma_f16_ss_pair(dacc, ad, bd, idesc, acc);
                            else
                                mma_f16_ss(dacc, ad, bd, idesc, acc);
                        }
                    if (CG == 2)
                        mma_commit_pair_both(&empty[s]);
                    else
                        mma_commit(&empty[s]);
                }
                if (ok) {
                    if (CG == 2)
                        mma_commit_pair_both(&tfull[buf]);
                    else
                        mma_commit(&tfull[buf]);
                }
            }
            // all issued MMAs complete before either CTA may release TMEM or leave
            if (CG == 2)
                mma_commit_pair_local(mma_done);
            else
                mma_commit(mma_done);
            volatile int dummy = 0;
            mbar_wait(mma_done, 0, &dummy, kDevTimeoutMma, p.err);
        }
    } else {
        // ------------------------------------------------ epilogue (warps 0-7)
        const int quarter = warp & 3;
        const int grp = warp >> 2;
        const int r = quarter * 32 + lane;
        if constexpr (epi_resid<EPI>()) {
            resid_epilogue<BN, AMODE, CG, C::RING_BUFS>(p, tmem_base, tfull, tempty, tempty_c,
                                                      ring_bars + warp * C::RING_BUFS,
                                                      epi_stage + warp * 4096 * C::RING_BUFS, &mapC0, &mapC1,
                                                      abort_flag, abort_pair, quarter, grp, lane, rank, unit,
                                                      num_units, num_tiles);
        } else {
            const RowStage st{epi_stage + warp * 4096, lane};
            const StoreMaps maps{{&mapC0, &mapC1, &mapC2}};
            uint32_t tcount = 0, h4count = 0;
            for (int t = unit; t < num_tiles; t += num_units, ++tcount) {
                const uint32_t buf = tcount & 1;
                const uint32_t tph = (tcount >> 1) & 1;
                const TileGeom g = tile_geom<AMODE, CG>(p, t, rank);
                if (!mbar_wait(&tfull[buf], tph, abort_flag, kDevTimeoutEpilogue, p.err)) {
                    abort_pair();
                    break;
                }
                tc_fence_after();
                if (g.live) {
                    const uint32_t tacc =
                        tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * C::ACC_COLS;
                    const Head4Sync h4{head4_part, head4_wts, h4_full, h4_empty, abort_flag, h4count++};
                    epilogue_tile<T, BN, AMODE, EPI>(p, g, tacc, r, grp, h4, st, maps);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    if (CG == 2)
                        mbar_arrive_cluster(tempty_c + buf * 8);
                    else
                        mbar_arrive(&tempty[buf]);
                }
            }
        }
        if (lane == 0) bulk_wait_all();  // TMA stores of this warp complete before the CTA ends
    }
    __syncwarp();
    if (CG == 2)
        cluster_sync();  // no CTA leaves while its peer may still signal or read it
    else
        __syncthreads();
    if (warp == kGemmMmaWarp) {
        tc_fence_after();
        if (CG == 2)
            tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
        else
            tmem_dealloc(tmem_base, C::TMEM_COLS);
    }
}

}  // namespace m3r
