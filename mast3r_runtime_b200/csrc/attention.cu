// Non-causal flash attention on tcgen05 (sm_100a), head dim 64, 16-bit (fp16 or
// bf16) in/out, fp32 softmax statistics and accumulation.
//
//   Q, K, V : head-major [seq, head, tok, 64] (written by the QKV GEMM epilogue)
//   O       : token-major [seq, tok, head * 64] (the A operand of the output projection)
//
// One CTA = 128 query rows of one (seq, head), two CTAs per SM.  320 threads:
// warps 0-7 softmax, warp 8 TMA producer, warp 9 MMA issuer.  Each query row (TMEM
// lane) is shared by two softmax threads, warp w and warp w + 4 (same TMEM lane
// quarter): thread half h takes keys [64 h, 64 h + 64) of every tile and output
// columns [32 h, 32 h + 32), which halves the per-thread softmax latency of a tile.
// The two halves agree on the row maximum through shared memory each tile and add
// their row sums once at the end.
// TMEM (256 columns per CTA): S = Q K^T in [0,128), P (two 16-bit values per
// column) in [128,192), O in [192,256).  S uses an SS MMA; O += P V uses a TS MMA
// with P from TMEM and V read MN-major straight from its TMA tile.  K and V tiles of
// 128 keys stream through separate rings, so a K stage is refilled as soon as its
// Q K^T has run; keys beyond Nk are masked to -inf (their V rows are zero-filled by
// TMA).  Scores never touch HBM.
//
// Semantics: softmax(Q K^T * scale) V per head, as
// backends/python/croco_encoder.py:80-85 and croco_decoder.py:76-82, 171-177.
#include <cmath>
#include <mutex>

#include "attention.h"
#include "common.cuh"

namespace m3r {

namespace {

constexpr int kTile = 128;
constexpr int kTileBytes = kTile * 64 * 2;  // 16 KB: 128 rows x 128 bytes
constexpr int kKStages = 2;                 // K ring (a stage frees when its Q K^T has run)
constexpr int kVStages = 3;                 // V ring (a stage frees when its P V has run)
constexpr int kSoftmaxWarps = 8;
constexpr int kSoftmaxThreads = kSoftmaxWarps * 32;
constexpr int kProducerWarp = kSoftmaxWarps;
constexpr int kMmaWarp = kSoftmaxWarps + 1;
constexpr int kThreads = (kSoftmaxWarps + 2) * 32;
// shared memory: Q | K ring | V ring | row-maximum exchange [2 parities][2 halves][128]
// | row-sum exchange [2 halves][128] | barriers.  The dynamic shared memory base is
// 1024-byte aligned (declared alignment, checked at run time), so two CTAs fit in
// one SM with their 1 KB reserves.
constexpr int kXmOff = (1 + kKStages + kVStages) * kTileBytes;
constexpr int kXlOff = kXmOff + 2 * 2 * kTile * 4;
constexpr int kBarOff = kXlOff + 2 * kTile * 4;
constexpr int kSmemBytes = kBarOff + 256;
constexpr uint32_t kColS = 0, kColP = 128, kColO = 192, kTmemCols = 256;

// fp16 operands take the packed fp16 exponential path of the softmax; bf16 keeps
// fp32 exponentials (an 8-bit significand for the exponent would cost ~0.5% on P).
template <class T>
constexpr bool kHalfExp = false;
template <>
constexpr bool kHalfExp<__half> = true;

#ifndef M3R_ATTN_POLY_PAIRS_F16
#define M3R_ATTN_POLY_PAIRS_F16 4
#endif
#ifndef M3R_ATTN_POLY_PAIRS_BF16
#define M3R_ATTN_POLY_PAIRS_BF16 4
#endif
template <class T>
constexpr int kPolyPairs = M3R_ATTN_POLY_PAIRS_BF16;
template <>
constexpr int kPolyPairs<__half> = M3R_ATTN_POLY_PAIRS_F16;

// the 16-bit pattern layout: mantissa bits and exponent bias + 0.5
template <class T>
struct Bits16;
template <>
struct Bits16<__half> {
    static constexpr float kScale = 1024.0f, kBias = 15.5f, kMin = -15.5f;  // 2^(v+0.5) < 2^-14 -> (near) 0
};
template <>
struct Bits16<__nv_bfloat16> {
    static constexpr float kScale = 128.0f, kBias = 127.5f, kMin = -60.0f;
};
constexpr float kShifter = 12582912.0f;  // 1.5 * 2^23: x + kShifter rounds x to an integer
constexpr float kG0 = -0.085893214f, kG1 = -0.01980106f, kG2 = 0.3431447f, kG3 = 0.07920424f;

__device__ __forceinline__ float max3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// (a, b) * s + t in one fma.rn.f32x2
__device__ __forceinline__ float2 fma2(float a, float b, float s, float t) {
    unsigned long long ab, ss, tt, r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(ab) : "f"(a), "f"(b));
    asm("mov.b64 %0, {%1, %1};" : "=l"(ss) : "f"(s));
    asm("mov.b64 %0, {%1, %1};" : "=l"(tt) : "f"(t));
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(ab), "l"(ss), "l"(tt));
    float2 o;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(o.x), "=f"(o.y) : "l"(r));
    return o;
}

__device__ __forceinline__ unsigned long long pk2(float a, float b) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ unsigned long long fma2v(unsigned long long a, unsigned long long b, unsigned long long c) {
    unsigned long long r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ unsigned long long add2v(unsigned long long a, unsigned long long b) {
    unsigned long long r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ unsigned long long sub2v(unsigned long long a, unsigned long long b) {
    unsigned long long r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

// 16-bit pair (low half first) of 2^(s0 * sl2 - mh + 0.5), 2^(s1 * sl2 - mh + 0.5) on
// the FMA pipe (see the comment on kPolyPairs); mh = the row's offset + 0.5.
template <class T>
__device__ __forceinline__ uint32_t exp2_poly2(float s0, float s1, float sl2, float mh) {
    float v0, v1;
    {
        const unsigned long long v = fma2v(pk2(s0, s1), pk2(sl2, sl2), pk2(-mh, -mh));
        asm("mov.b64 {%0, %1}, %2;" : "=f"(v0), "=f"(v1) : "l"(v));
    }
    v0 = fmaxf(v0, Bits16<T>::kMin);
    v1 = fmaxf(v1, Bits16<T>::kMin);
    const unsigned long long v = pk2(v0, v1);
    const unsigned long long sh = pk2(kShifter, kShifter);
    const unsigned long long n = sub2v(add2v(v, sh), sh);  // round(v)
    const unsigned long long f = sub2v(v, n);               // in [-0.5, 0.5]
    unsigned long long q = fma2v(f, pk2(kG3, kG3), pk2(kG2, kG2));
    q = fma2v(q, f, pk2(kG1, kG1));
    q = fma2v(q, f, pk2(kG0, kG0));                         // g(f + 0.5)
    const unsigned long long t = add2v(v, q);
    constexpr float kC = kShifter + Bits16<T>::kScale * Bits16<T>::kBias;
    const unsigned long long y = fma2v(t, pk2(Bits16<T>::kScale, Bits16<T>::kScale), pk2(kC, kC));
    uint32_t y0, y1;
    asm("mov.b64 {%0, %1}, %2;" : "=r"(y0), "=r"(y1) : "l"(y));
    return __byte_perm(y0, y1, 0x5410);  // low 16 bits of each
}

// fp16 pair (low half = x0) of 2^x0, 2^x1
__device__ __forceinline__ uint32_t ex2_h2(float x0, float x1) {
    const __half2 h = __floats2half2_rn(x0, x1);
    uint32_t e;
    asm("ex2.approx.f16x2 %0, %1;" : "=r"(e) : "r"(*reinterpret_cast<const uint32_t*>(&h)));
    return e;
}

// s0 += low fp16 of h, s1 += high fp16 of h (fp32 accumulation)
__device__ __forceinline__ void add_h2_f32(float& s0, float& s1, uint32_t h) {
    asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
        "add.f32.f16 %0, lo, %0;\n\tadd.f32.f16 %1, hi, %1;\n\t}"
        : "+f"(s0), "+f"(s1)
        : "r"(h));
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]));
}

struct AttnParams {
    int nq, nk, heads, n_kv_tiles;
    float scale_log2;  // scale * log2(e)
    void* out;
    int* err;          // device status word (bounded-wait timeouts)
};

template <class T>
__global__ void __launch_bounds__(kThreads, 2)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap mapQ, const __grid_constant__ CUtensorMap mapK,
                    const __grid_constant__ CUtensorMap mapV, const __grid_constant__ AttnParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    if ((smem_u32(smem) & 1023u) != 0) {  // 128-byte swizzled tiles need 1024-byte alignment
        if (threadIdx.x == 0) atomicCAS(p.err, 0, kDevBadSmemAlign);
        return;
    }
    uint8_t* sQ = smem;
    uint8_t* sK = smem + kTileBytes;                   // kKStages
    uint8_t* sV = smem + (1 + kKStages) * kTileBytes;  // kVStages
    float* xm = reinterpret_cast<float*>(smem + kXmOff);  // [parity][half][row] partial row maxima
    float* xl = reinterpret_cast<float*>(smem + kXlOff);  // [half][row] partial row sums
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBarOff);
    uint64_t* q_full = bars + 0;
    uint64_t* k_full = bars + 1;                         // [kKStages]
    uint64_t* k_empty = k_full + kKStages;               // [kKStages]
    uint64_t* v_full = k_empty + kKStages;               // [kVStages]
    uint64_t* v_empty = v_full + kVStages;               // [kVStages]
    uint64_t* s_full = v_empty + kVStages;
    uint64_t* s_empty = s_full + 1;
    uint64_t* p_full = s_full + 2;
    uint64_t* o_done = s_full + 3;
    uint64_t* mma_done = s_full + 4;
    uint64_t* xm_bar = s_full + 5;   // all softmax threads published their tile maxima
    uint64_t* xl_bar = s_full + 6;   // all softmax threads published their row sums
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_full + 7);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int q0 = blockIdx.x * kTile;
    const int head = blockIdx.y;
    const int seq = blockIdx.z;
    const int plane = seq * p.heads + head;
    const int nkv = p.n_kv_tiles;

    if (warp == kProducerWarp && lane == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < kKStages; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
        }
        for (int s = 0; s < kVStages; ++s) {
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
        }
        mbar_init(s_full, 1);
        mbar_init(s_empty, kSoftmaxThreads);
        mbar_init(p_full, kSoftmaxThreads);
        mbar_init(o_done, 1);
        mbar_init(mma_done, 1);
        mbar_init(xm_bar, kSoftmaxThreads);
        mbar_init(xl_bar, kSoftmaxThreads);
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tmap(&mapQ);
        prefetch_tmap(&mapK);
        prefetch_tmap(&mapV);
    }
    if (warp == kMmaWarp) tmem_alloc(tmem_slot, kTmemCols);
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == kProducerWarp) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            mbar_arrive_expect_tx(q_full, kTileBytes);
            tma_load_3d(sQ, &mapQ, q_full, 0, q0, plane);
            int k_issued = 0, v_issued = 0;
            bool ok = true;
            for (int j = 0; j < nkv && ok; ++j) {
                const int sk = j % kKStages, sv = j % kVStages;
                if (!mbar_wait(&k_empty[sk], ((j / kKStages) & 1) ^ 1, abort_flag, kDevTimeoutProducer, p.err)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&k_full[sk], kTileBytes);
                tma_load_3d(sK + sk * kTileBytes, &mapK, &k_full[sk], 0, j * kTile, plane);
                k_issued = j + 1;
                if (!mbar_wait(&v_empty[sv], ((j / kVStages) & 1) ^ 1, abort_flag, kDevTimeoutProducer, p.err)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&v_full[sv], kTileBytes);
                tma_load_3d(sV + sv * kTileBytes, &mapV, &v_full[sv], 0, j * kTile, plane);
                v_issued = j + 1;
            }
            if (!ok) {
                // drain: wait (bounded) for loads that may still be in flight
                volatile int dummy = 0;
                mbar_wait(q_full, 0, &dummy, kDevTimeoutProducer, p.err);
                for (int j = k_issued > kKStages ? k_issued - kKStages : 0; j < k_issued; ++j)
                    mbar_wait(&k_full[j % kKStages], (j / kKStages) & 1, &dummy, kDevTimeoutProducer, p.err);
                for (int j = v_issued > kVStages ? v_issued - kVStages : 0; j < v_issued; ++j)
                    mbar_wait(&v_full[j % kVStages], (j / kVStages) & 1, &dummy, kDevTimeoutProducer, p.err);
            }
        }
    } else if (warp == kMmaWarp) {
        // ------------------------------------------------------------ MMA issuer
        // S_{j+1} = Q K_{j+1}^T is issued as soon as the softmax threads have read S_j
        // into registers, so it overlaps their exponentials; O += P_j V_j follows P_j.
        if (lane == 0) {
            constexpr uint32_t idesc_s = idesc_f16kind<T>(128, 128, false, false);
            constexpr uint32_t idesc_o = idesc_f16kind<T>(128, 64, false, true);
            const uint32_t q_addr = smem_u32(sQ);
            auto issue_s = [&](int j) {
                const uint32_t k_addr = smem_u32(sK + (j % kKStages) * kTileBytes);
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    mma_f16_ss(tmem + kColS, umma_desc_sw128(q_addr + k * 32, 16, 1024),
                               umma_desc_sw128(k_addr + k * 32, 16, 1024), idesc_s, k > 0 ? 1u : 0u);
                mma_commit(s_full);
                mma_commit(&k_empty[j % kKStages]);
            };
            bool ok = mbar_wait(q_full, 0, abort_flag, kDevTimeoutMma, p.err) &&
                      mbar_wait(&k_full[0], 0, abort_flag, kDevTimeoutMma, p.err);
            if (ok) {
                tc_fence_after();
                issue_s(0);
            }
            for (int j = 0; j < nkv && ok; ++j) {
                if (j + 1 < nkv) {
                    if (!mbar_wait(&k_full[(j + 1) % kKStages], ((j + 1) / kKStages) & 1, abort_flag, kDevTimeoutMma,
                                   p.err) ||
                        !mbar_wait(s_empty, j & 1, abort_flag, kDevTimeoutMma, p.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    issue_s(j + 1);
                }
                if (!mbar_wait(&v_full[j % kVStages], (j / kVStages) & 1, abort_flag, kDevTimeoutMma, p.err) ||
                    !mbar_wait(p_full, j & 1, abort_flag, kDevTimeoutMma, p.err)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t v_addr = smem_u32(sV + (j % kVStages) * kTileBytes);
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    mma_f16_ts(tmem + kColO, tmem + kColP + k * 8, umma_desc_sw128(v_addr + k * 2048, 16384, 1024),
                               idesc_o, (j > 0 || k > 0) ? 1u : 0u);
                mma_commit(&v_empty[j % kVStages]);
                mma_commit(o_done);
            }
            mma_commit(mma_done);
            volatile int dummy = 0;
            mbar_wait(mma_done, 0, &dummy, kDevTimeoutMma, p.err);
        }
    } else {
        // ------------------------------------------------------------ softmax (warps 0-7)
        // Lazy rescaling: the exponent offset m_use only moves when the row maximum
        // exceeds it by more than 8 (log2 units), so P <= 2^8 and O is rescaled rarely.
        // Both halves of a row take the same decisions (same maxima, same order).
        const int quarter = warp & 3, half = warp >> 2;
        const int r = quarter * 32 + lane;
        const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
        const uint32_t tS = tmem + lane_base + kColS + 64 * half;
        const uint32_t tP = tmem + lane_base + kColP + 32 * half;
        const uint32_t tO = tmem + lane_base + kColO + 32 * half;
        const float sl2 = p.scale_log2;
        float m_use = -INFINITY, l_run = 0.0f;
        bool ok = true;
        for (int j = 0; j < nkv; ++j) {
            if (!mbar_wait(s_full, j & 1, abort_flag, kDevTimeoutSoftmax, p.err)) { ok = false; break; }
            tc_fence_after();
            uint32_t v[2][32];
            tmem_ld32(tS, v[0]);
            tmem_ld32(tS + 32, v[1]);
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(s_empty);  // S is in registers: the next S may overwrite it
            const int valid = p.nk - j * kTile - 64 * half;  // keys of this half that exist (may be <= 0)
            const bool full_half = valid >= 64;
            // partial row maximum over this half, 8 independent chains
            float mp[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) mp[u] = -INFINITY;
            if (full_half) {
#pragma unroll
                for (int c = 0; c < 2; ++c)
#pragma unroll
                    for (int i = 0; i < 32; i += 2) {
                        float& m = mp[(c * 16 + i / 2) & 7];
                        m = max3(m, __uint_as_float(v[c][i]), __uint_as_float(v[c][i + 1]));
                    }
            } else {
#pragma unroll
                for (int c = 0; c < 2; ++c)
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (c * 32 + i < valid) mp[i & 7] = fmaxf(mp[i & 7], __uint_as_float(v[c][i]));
            }
            const float pmax = max3(max3(mp[0], mp[1], mp[2]), max3(mp[3], mp[4], mp[5]), fmaxf(mp[6], mp[7]));
            // exchange with the other half of the row (parity-buffered slots: a slot is
            // rewritten two tiles later, after the partner has passed the next exchange)
            float* slot = xm + (j & 1) * 2 * kTile;
            slot[half * kTile + r] = pmax;
            mbar_arrive(xm_bar);
            if (!mbar_wait(xm_bar, j & 1, abort_flag, kDevTimeoutSoftmax, p.err)) { ok = false; break; }
            const float mx = fmaxf(slot[r], slot[kTile + r]);  // same operand order in both halves
            const float m_cand = mx * sl2;
            const float m_new = (m_cand > m_use + 8.0f) ? m_cand : m_use;
            const float alpha = ex2_approx(m_use - m_new);  // 1 when m_use is kept, 0 on the first tile
            float rowsum = 0.0f;
            uint32_t pk[2][16];
            if (kHalfExp<T> && full_half) {
                // fp16 operands: the exponent x = s * scale * log2(e) - m is formed in fp32
                // (two lanes per fma.rn.f32x2), rounded to fp16 and exponentiated two at a
                // time (ex2.approx.f16x2), which yields P already packed for the PV MMA;
                // the row sum accumulates the fp16 P values in fp32.
                float rs[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) rs[u] = 0.0f;
#pragma unroll
                for (int c = 0; c < 2; ++c)
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        if (i < kPolyPairs<T>) {
                            pk[c][i] = exp2_poly2<T>(__uint_as_float(v[c][2 * i]), __uint_as_float(v[c][2 * i + 1]), sl2, m_new + 0.5f);
                        } else {
                            const float2 x = fma2(__uint_as_float(v[c][2 * i]), __uint_as_float(v[c][2 * i + 1]), sl2, -m_new);
                            pk[c][i] = ex2_h2(x.x, x.y);
                        }
                        const int u = 2 * (i & 3);
                        add_h2_f32(rs[u], rs[u + 1], pk[c][i]);
                    }
                rowsum = ((rs[0] + rs[1]) + (rs[2] + rs[3])) + ((rs[4] + rs[5]) + (rs[6] + rs[7]));
            } else {
                float rs[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) rs[u] = 0.0f;
#pragma unroll
                for (int c = 0; c < 2; ++c)
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int c0 = c * 32 + 2 * i;
                        if (full_half && i < kPolyPairs<T>) {  // bf16: exponentials on the FMA pipe
                            pk[c][i] = exp2_poly2<T>(__uint_as_float(v[c][2 * i]), __uint_as_float(v[c][2 * i + 1]), sl2,
                                                     m_new + 0.5f);
                            const float2 pf = Elem<T>::unpack(pk[c][i]);
                            rs[2 * (i & 3)] += pf.x;
                            rs[2 * (i & 3) + 1] += pf.y;
                            continue;
                        }
                        float p0 = ex2_approx(__uint_as_float(v[c][2 * i]) * sl2 - m_new);
                        float p1 = ex2_approx(__uint_as_float(v[c][2 * i + 1]) * sl2 - m_new);
                        if (!full_half) {
                            p0 = c0 < valid ? p0 : 0.0f;
                            p1 = c0 + 1 < valid ? p1 : 0.0f;
                        }
                        rs[2 * (i & 3)] += p0;
                        rs[2 * (i & 3) + 1] += p1;
                        pk[c][i] = Elem<T>::pack(p0, p1);
                    }
                rowsum = ((rs[0] + rs[1]) + (rs[2] + rs[3])) + ((rs[4] + rs[5]) + (rs[6] + rs[7]));
            }
            if (j > 0) {
                // P buffer free and O stable once PV of the previous tile is done
                if (!mbar_wait(o_done, (j - 1) & 1, abort_flag, kDevTimeoutSoftmax, p.err)) { ok = false; break; }
                tc_fence_after();
                if (__any_sync(0xffffffffu, alpha != 1.0f)) {
                    uint32_t o[32];
                    tmem_ld32(tO, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                    tmem_st32(tO, o);
                }
            }
            tmem_st16(tP, pk[0]);
            tmem_st16(tP + 16, pk[1]);
            tmem_wait_st();
            l_run = l_run * alpha + rowsum;
            m_use = m_new;
            tc_fence_before();
            mbar_arrive(p_full);
        }
        // row sum: this half's share + the other half's
        xl[half * kTile + r] = l_run;
        mbar_arrive(xl_bar);
        if (ok && mbar_wait(xl_bar, 0, abort_flag, kDevTimeoutSoftmax, p.err) &&
            mbar_wait(o_done, (nkv - 1) & 1, abort_flag, kDevTimeoutSoftmax, p.err)) {
            tc_fence_after();
            uint32_t o[32];
            tmem_ld32(tO, o);
            tmem_wait_ld();
            const int q = q0 + r;
            if (q < p.nq) {
                const float inv = 1.0f / (xl[r] + xl[kTile + r]);  // same operand order in both halves
                T* dst = reinterpret_cast<T*>(p.out) + (static_cast<long long>(seq) * p.nq + q) * (p.heads * 64) +
                         head * 64 + 32 * half;
                uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
                for (int qq = 0; qq < 4; ++qq) {
                    uint4 u;
                    u.x = Elem<T>::pack(__uint_as_float(o[qq * 8 + 0]) * inv, __uint_as_float(o[qq * 8 + 1]) * inv);
                    u.y = Elem<T>::pack(__uint_as_float(o[qq * 8 + 2]) * inv, __uint_as_float(o[qq * 8 + 3]) * inv);
                    u.z = Elem<T>::pack(__uint_as_float(o[qq * 8 + 4]) * inv, __uint_as_float(o[qq * 8 + 5]) * inv);
                    u.w = Elem<T>::pack(__uint_as_float(o[qq * 8 + 6]) * inv, __uint_as_float(o[qq * 8 + 7]) * inv);
                    d4[qq] = u;
                }
            }
        }
    }
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

template <class T>
void launch(cudaStream_t s, const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const AttnParams& p,
            dim3 grid) {
    static std::once_flag once;
    std::call_once(once, [] {
        int ndev = 0, cur = 0;
        M3R_CUDA(cudaGetDeviceCount(&ndev));
        M3R_CUDA(cudaGetDevice(&cur));
        for (int d = 0; d < ndev; ++d) {
            M3R_CUDA(cudaSetDevice(d));
            M3R_CUDA(cudaFuncSetAttribute(attn_fwd_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
        }
        M3R_CUDA(cudaSetDevice(cur));
    });
    attn_fwd_kernel<T><<<grid, kThreads, kSmemBytes, s>>>(mq, mk, mv, p);
    M3R_CUDA(cudaGetLastError());
}

}  // namespace

void attention_fwd(cudaStream_t s, int dt, const void* q, const void* k, const void* v, void* out, int n_seq,
                   int heads, int nq, int nk, float scale, int* err) {
    M3R_REQUIRE(n_seq > 0 && heads > 0 && nq > 0 && nk > 0, "attention: bad shape");
    M3R_REQUIRE(n_seq <= 65535 && heads <= 65535, "attention: grid too large");
    const CUtensorMap mq = tmap_3d_rows64(dt, q, nq, static_cast<uint64_t>(n_seq) * heads, kTile);
    const CUtensorMap mk = tmap_3d_rows64(dt, k, nk, static_cast<uint64_t>(n_seq) * heads, kTile);
    const CUtensorMap mv = tmap_3d_rows64(dt, v, nk, static_cast<uint64_t>(n_seq) * heads, kTile);
    AttnParams p;
    p.nq = nq;
    p.nk = nk;
    p.heads = heads;
    p.n_kv_tiles = (nk + kTile - 1) / kTile;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.out = out;
    p.err = err;
    const dim3 grid((nq + kTile - 1) / kTile, heads, n_seq);
    if (dt == DT_F16)
        launch<__half>(s, mq, mk, mv, p, grid);
    else if (dt == DT_BF16)
        launch<__nv_bfloat16>(s, mq, mk, mv, p, grid);
    else
        throw Error(kErrArg, "attention: unknown operand type");
}

}  // namespace m3r
