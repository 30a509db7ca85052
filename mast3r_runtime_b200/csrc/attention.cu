// Non-causal flash attention on tcgen05 (sm_100a), head dim 64, 16-bit (fp16 or
// bf16) in/out, fp32 softmax statistics and accumulation.
//
//   Q, K, V : head-major [seq, head, tok, 64] (written by the QKV GEMM epilogue)
//   O       : token-major [seq, tok, head * 64] (the A operand of the output projection)
//
// One CTA = 128 query rows of one (seq, head).  192 threads: warps 0-3 softmax
// (thread = query row = TMEM lane), warp 4 TMA producer, warp 5 MMA issuer.
// TMEM (256 columns, so two CTAs fit on an SM): S = Q K^T in [0,128), P (two
// 16-bit values per column) in [128,192), O in [192,256).  S uses an SS MMA;
// O += P V uses a TS MMA with P from TMEM and V read MN-major straight from its
// TMA tile.  K/V tiles of 128 keys are double-buffered; keys beyond Nk are masked
// to -inf (their V rows are zero-filled by TMA).  Scores never touch HBM.
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
constexpr int kSmemBytes = 5 * kTileBytes + 1024 + 256;
constexpr uint32_t kColS = 0, kColP = 128, kColO = 192, kTmemCols = 256;

// fp16 operands take the packed fp16 exponential path of the softmax; bf16 keeps
// fp32 exponentials (an 8-bit significand for the exponent would cost ~0.5% on P).
template <class T>
constexpr bool kHalfExp = false;
template <>
constexpr bool kHalfExp<__half> = true;

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

struct AttnParams {
    int nq, nk, heads, n_kv_tiles;
    float scale_log2;  // scale * log2(e)
    void* out;
    int* err;          // device status word (bounded-wait timeouts)
};

template <class T>
__global__ void __launch_bounds__(192, 2)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap mapQ, const __grid_constant__ CUtensorMap mapK,
                    const __grid_constant__ CUtensorMap mapV, const __grid_constant__ AttnParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;
    uint8_t* sK = smem + kTileBytes;       // 2 stages
    uint8_t* sV = smem + 3 * kTileBytes;   // 2 stages
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 5 * kTileBytes);
    uint64_t* q_full = bars + 0;
    uint64_t* kv_full = bars + 1;   // [2]
    uint64_t* kv_empty = bars + 3;  // [2]
    uint64_t* s_full = bars + 5;
    uint64_t* s_empty = bars + 6;
    uint64_t* p_full = bars + 7;
    uint64_t* o_done = bars + 8;
    uint64_t* mma_done = bars + 9;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int q0 = blockIdx.x * kTile;
    const int head = blockIdx.y;
    const int seq = blockIdx.z;
    const int plane = seq * p.heads + head;
    const int nkv = p.n_kv_tiles;

    if (warp == 4 && lane == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        mbar_init(s_full, 1);
        mbar_init(s_empty, 128);
        mbar_init(p_full, 128);
        mbar_init(o_done, 1);
        mbar_init(mma_done, 1);
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tmap(&mapQ);
        prefetch_tmap(&mapK);
        prefetch_tmap(&mapV);
    }
    if (warp == 5) tmem_alloc(tmem_slot, kTmemCols);
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 4) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            mbar_arrive_expect_tx(q_full, kTileBytes);
            tma_load_3d(sQ, &mapQ, q_full, 0, q0, plane);
            int issued = 0;
            bool ok = true;
            for (int j = 0; j < nkv; ++j) {
                const int st = j & 1;
                const uint32_t ph = (j >> 1) & 1;
                if (!mbar_wait(&kv_empty[st], ph ^ 1, abort_flag, kDevTimeoutProducer, p.err)) { ok = false; break; }
                mbar_arrive_expect_tx(&kv_full[st], 2 * kTileBytes);
                tma_load_3d(sK + st * kTileBytes, &mapK, &kv_full[st], 0, j * kTile, plane);
                tma_load_3d(sV + st * kTileBytes, &mapV, &kv_full[st], 0, j * kTile, plane);
                issued = j + 1;
            }
            if (!ok) {
                volatile int dummy = 0;
                mbar_wait(q_full, 0, &dummy, kDevTimeoutProducer, p.err);
                for (int j = issued > 2 ? issued - 2 : 0; j < issued; ++j)
                    mbar_wait(&kv_full[j & 1], (j >> 1) & 1, &dummy, kDevTimeoutProducer, p.err);
            }
        }
    } else if (warp == 5) {
        // ------------------------------------------------------------ MMA issuer
        // S_{j+1} = Q K_{j+1}^T is issued as soon as the softmax warps have read S_j
        // into registers, so it overlaps their exponentials; O += P_j V_j follows P_j.
        if (lane == 0) {
            constexpr uint32_t idesc_s = idesc_f16kind<T>(128, 128, false, false);
            constexpr uint32_t idesc_o = idesc_f16kind<T>(128, 64, false, true);
            const uint32_t q_addr = smem_u32(sQ);
            auto issue_s = [&](int j) {
                const uint32_t k_addr = smem_u32(sK + (j & 1) * kTileBytes);
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    mma_f16_ss(tmem + kColS, umma_desc_sw128(q_addr + k * 32, 16, 1024),
                               umma_desc_sw128(k_addr + k * 32, 16, 1024), idesc_s, k > 0 ? 1u : 0u);
                mma_commit(s_full);
            };
            bool ok = mbar_wait(q_full, 0, abort_flag, kDevTimeoutMma, p.err) &&
                      mbar_wait(&kv_full[0], 0, abort_flag, kDevTimeoutMma, p.err);
            if (ok) {
                tc_fence_after();
                issue_s(0);
            }
            for (int j = 0; j < nkv && ok; ++j) {
                if (j + 1 < nkv) {
                    if (!mbar_wait(&kv_full[(j + 1) & 1], ((j + 1) >> 1) & 1, abort_flag, kDevTimeoutMma, p.err) ||
                        !mbar_wait(s_empty, j & 1, abort_flag, kDevTimeoutMma, p.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    issue_s(j + 1);
                }
                if (!mbar_wait(p_full, j & 1, abort_flag, kDevTimeoutMma, p.err)) { ok = false; break; }
                tc_fence_after();
                const uint32_t v_addr = smem_u32(sV + (j & 1) * kTileBytes);
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    mma_f16_ts(tmem + kColO, tmem + kColP + k * 8, umma_desc_sw128(v_addr + k * 2048, 16384, 1024),
                               idesc_o, (j > 0 || k > 0) ? 1u : 0u);
                mma_commit(&kv_empty[j & 1]);
                mma_commit(o_done);
            }
            mma_commit(mma_done);
            volatile int dummy = 0;
            mbar_wait(mma_done, 0, &dummy, kDevTimeoutMma, p.err);
        }
    } else {
        // ------------------------------------------------------------ softmax (warps 0-3)
        // Lazy rescaling: the exponent offset m_use only moves when the row maximum
        // exceeds it by more than 8 (log2 units), so P <= 2^8 and O is rescaled rarely.
        const int r = warp * 32 + lane;
        const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
        const uint32_t tS = tmem + lane_base + kColS;
        const uint32_t tP = tmem + lane_base + kColP;
        const uint32_t tO = tmem + lane_base + kColO;
        const float sl2 = p.scale_log2;
        float m_use = -INFINITY, l_run = 0.0f;
        bool ok = true;
        for (int j = 0; j < nkv; ++j) {
            if (!mbar_wait(s_full, j & 1, abort_flag, kDevTimeoutSoftmax, p.err)) { ok = false; break; }
            tc_fence_after();
            uint32_t v[4][32];
#pragma unroll
            for (int c = 0; c < 4; ++c) tmem_ld32(tS + c * 32, v[c]);
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(s_empty);  // S is in registers: the next S may overwrite it
            const int valid = p.nk - j * kTile;  // keys valid in this tile (>= 1)
            const bool full_tile = valid >= kTile;
            // row maximum as 8 independent partial maxima (short dependency chains)
            float mp[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) mp[u] = -INFINITY;
            if (full_tile) {
#pragma unroll
                for (int c = 0; c < 4; ++c)
#pragma unroll
                    for (int i = 0; i < 32; i += 2) {
                        float& m = mp[(c * 16 + i / 2) & 7];
                        m = max3(m, __uint_as_float(v[c][i]), __uint_as_float(v[c][i + 1]));
                    }
            } else {
#pragma unroll
                for (int c = 0; c < 4; ++c)
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (c * 32 + i < valid) mp[i & 7] = fmaxf(mp[i & 7], __uint_as_float(v[c][i]));
            }
            const float mx = max3(max3(mp[0], mp[1], mp[2]), max3(mp[3], mp[4], mp[5]), fmaxf(mp[6], mp[7]));
            const float m_cand = mx * sl2;
            const float m_new = (m_cand > m_use + 8.0f) ? m_cand : m_use;
            const float alpha = ex2_approx(m_use - m_new);  // 1 when m_use is kept, 0 on the first tile
            float rowsum = 0.0f;
            uint32_t pk[4][16];
            if (kHalfExp<T> && full_tile) {
                // fp16 operands: the exponent x = s * scale * log2(e) - m is formed in fp32
                // (two lanes per fma.rn.f32x2), rounded to fp16 and exponentiated two at a
                // time (ex2.approx.f16x2), which yields P already packed for the PV MMA and
                // halves the MUFU work; the row sum accumulates the fp16 P values in fp32.
                float rs[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) rs[u] = 0.0f;
#pragma unroll
                for (int c = 0; c < 4; ++c)
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float2 x = fma2(__uint_as_float(v[c][2 * i]), __uint_as_float(v[c][2 * i + 1]), sl2, -m_new);
                        pk[c][i] = ex2_h2(x.x, x.y);
                        const int u = 2 * (i & 3);
                        add_h2_f32(rs[u], rs[u + 1], pk[c][i]);
                    }
                rowsum = ((rs[0] + rs[1]) + (rs[2] + rs[3])) + ((rs[4] + rs[5]) + (rs[6] + rs[7]));
            } else {
                float rs[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) rs[u] = 0.0f;
#pragma unroll
                for (int c = 0; c < 4; ++c)
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int c0 = c * 32 + 2 * i;
                        float p0 = ex2_approx(__uint_as_float(v[c][2 * i]) * sl2 - m_new);
                        float p1 = ex2_approx(__uint_as_float(v[c][2 * i + 1]) * sl2 - m_new);
                        if (!full_tile) {
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
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        uint32_t o[32];
                        tmem_ld32(tO + c * 32, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                        tmem_st32(tO + c * 32, o);
                    }
                }
            }
#pragma unroll
            for (int c = 0; c < 4; ++c)
                asm volatile(
                    "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
                    "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(tP + c * 16),
                    "r"(pk[c][0]), "r"(pk[c][1]), "r"(pk[c][2]), "r"(pk[c][3]), "r"(pk[c][4]), "r"(pk[c][5]),
                    "r"(pk[c][6]), "r"(pk[c][7]), "r"(pk[c][8]), "r"(pk[c][9]), "r"(pk[c][10]), "r"(pk[c][11]),
                    "r"(pk[c][12]), "r"(pk[c][13]), "r"(pk[c][14]), "r"(pk[c][15]));
            tmem_wait_st();
            l_run = l_run * alpha + rowsum;
            m_use = m_new;
            tc_fence_before();
            mbar_arrive(p_full);
        }
        if (ok && mbar_wait(o_done, (nkv - 1) & 1, abort_flag, kDevTimeoutSoftmax, p.err)) {
            tc_fence_after();
            uint32_t o[2][32];
            tmem_ld32(tO, o[0]);
            tmem_ld32(tO + 32, o[1]);
            tmem_wait_ld();
            const int q = q0 + r;
            if (q < p.nq) {
                const float inv = 1.0f / l_run;
                T* dst = reinterpret_cast<T*>(p.out) + (static_cast<long long>(seq) * p.nq + q) * (p.heads * 64) + head * 64;
                uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int qq = 0; qq < 4; ++qq) {
                        uint4 u;
                        u.x = Elem<T>::pack(__uint_as_float(o[h][qq * 8 + 0]) * inv, __uint_as_float(o[h][qq * 8 + 1]) * inv);
                        u.y = Elem<T>::pack(__uint_as_float(o[h][qq * 8 + 2]) * inv, __uint_as_float(o[h][qq * 8 + 3]) * inv);
                        u.z = Elem<T>::pack(__uint_as_float(o[h][qq * 8 + 4]) * inv, __uint_as_float(o[h][qq * 8 + 5]) * inv);
                        u.w = Elem<T>::pack(__uint_as_float(o[h][qq * 8 + 6]) * inv, __uint_as_float(o[h][qq * 8 + 7]) * inv);
                        d4[h * 4 + qq] = u;
                    }
            }
        }
    }
    __syncthreads();
    if (warp == 5) {
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
    attn_fwd_kernel<T><<<grid, 192, kSmemBytes, s>>>(mq, mk, mv, p);
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
