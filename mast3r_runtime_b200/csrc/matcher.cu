// Reciprocal top-k descriptor matcher, bit-exact with the reference CPU matcher
// (csrc/cpu/matching.cpp:85-237 of the reference).
//
// Arithmetic is restated exactly as the reference computes it (its build has no
// FMA): normalisation s = s + x*x sequentially, n = sqrtf(s), x * (1.0f / n) when
// n > 1e-8; similarity d = d + a[k]*b[k] for k = 0..D-1, every multiply and add
// separately rounded (__fmul_rn / __fadd_rn, never contracted into an FMA).
// A packed mul.rn.f32x2 followed by add.rn.f32x2 is NOT safe for this: the
// pair was measured to be fused (about 60% of 24-term dot products changed),
// while packed/scalar mixes stay exact but are no faster than scalar here.
//
// Pipeline (one device, rows [row0, row1) of set A against all of set B):
//   normalize      one thread per row
//   argmax         128 x 128 tiles, 8 x 8 per thread; row and column maxima of
//                  every similarity (times conf_1[i] * conf_2[j] when confidence
//                  maps are given), fused -- the N x N matrix never exists.
//                  Partial maxima are merged with 64-bit atomicMax on keys
//                  (orderable(value) << 32) | (0xFFFFFFFF - index): the maximum
//                  key is the maximum value with the lowest index, which is the
//                  reference's strict-> first-wins rule.
//   candidates     reciprocal test nn_21[nn_12[i]] == i and sim >= threshold,
//                  compacted in ascending i (the reference's push_back order)
//   top-k          when more than top_k survive: radix select (16-bit digits) of
//                  the top_k largest (conf, -i) keys, then a bitonic sort of
//                  those, i.e. confidence descending, idx_1 ascending on ties.
#include <algorithm>
#include <type_traits>
#include <vector>

#include "matcher.h"
#include "tmap.h"

namespace m3r {

namespace {

__device__ __forceinline__ uint32_t orderable(float f) {
    if (f != f) return 0xFFFFFFFFu;  // NaN: only ever the seed of a row / column (see argmax_kernel)
    f = f + 0.0f;  // -0.0 -> +0.0: the reference's > comparison treats them as equal
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float from_orderable(uint32_t k) {
    const uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
    return __uint_as_float(u);
}

__device__ __forceinline__ unsigned long long make_key(float v, uint32_t idx) {
    return (static_cast<unsigned long long>(orderable(v)) << 32) | (0xFFFFFFFFu - idx);
}

// ------------------------------------------------------------------ normalize
// (in and out may be the same buffer: no __restrict__)
__global__ void normalize_kernel(const float* in, float* out, long long n, int d) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const float* r = in + i * d;
        float* o = out + i * d;
        float s = 0.0f;
        for (int k = 0; k < d; ++k) s = __fadd_rn(s, __fmul_rn(r[k], r[k]));
        s = sqrtf(s);
        if (s > 1e-8f) {
            const float inv = 1.0f / s;
            for (int k = 0; k < d; ++k) o[k] = __fmul_rn(r[k], inv);
        } else {
            for (int k = 0; k < d; ++k) o[k] = r[k];
        }
    }
}

// 24-channel rows as six 16-byte loads / stores per thread (rows of 96 bytes keep
// 16-byte alignment when the base is aligned); same operation order as above.
__global__ void normalize24_kernel(const float4* in, float4* out, long long n) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        float4 x[6];
#pragma unroll
        for (int q = 0; q < 6; ++q) x[q] = in[i * 6 + q];
        float s = 0.0f;
#pragma unroll
        for (int q = 0; q < 6; ++q) {
            s = __fadd_rn(s, __fmul_rn(x[q].x, x[q].x));
            s = __fadd_rn(s, __fmul_rn(x[q].y, x[q].y));
            s = __fadd_rn(s, __fmul_rn(x[q].z, x[q].z));
            s = __fadd_rn(s, __fmul_rn(x[q].w, x[q].w));
        }
        s = sqrtf(s);
        if (s > 1e-8f) {
            const float inv = 1.0f / s;
#pragma unroll
            for (int q = 0; q < 6; ++q) {
                x[q].x = __fmul_rn(x[q].x, inv);
                x[q].y = __fmul_rn(x[q].y, inv);
                x[q].z = __fmul_rn(x[q].z, inv);
                x[q].w = __fmul_rn(x[q].w, inv);
            }
        }
#pragma unroll
        for (int q = 0; q < 6; ++q) out[i * 6 + q] = x[q];
    }
}

// Both descriptor sets in one launch: a set is a few tens of MB, so one launch instead
// of two halves the ramp-up and tail.  A warp takes 32 consecutive rows of one set
// (3 KB): it loads them with coalesced 16-byte loads into shared memory, each lane
// normalises one row there (the sequential arithmetic of normalize24_kernel), and the
// warp stores the block back with coalesced 16-byte stores.
constexpr int kNormWarps = 8;
__global__ void __launch_bounds__(kNormWarps * 32)
    normalize24_pair_kernel(const float4* in1, float4* out1, long long n1, const float4* in2, float4* out2,
                            long long n2) {
    __shared__ float4 stage[kNormWarps][32 * 6];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    float4* sw = stage[w];
    const long long t1 = (n1 + 31) / 32, tasks = t1 + (n2 + 31) / 32;
    for (long long task = blockIdx.x * static_cast<long long>(kNormWarps) + w; task < tasks;
         task += static_cast<long long>(gridDim.x) * kNormWarps) {
        const bool first = task < t1;
        const long long r0 = 32 * (first ? task : task - t1);
        const long long n = first ? n1 : n2;
        const float4* in = (first ? in1 : in2) + r0 * 6;
        float4* out = (first ? out1 : out2) + r0 * 6;
        const int rows = n - r0 < 32 ? static_cast<int>(n - r0) : 32;
#pragma unroll
        for (int q = 0; q < 6; ++q) {
            const int f = lane + 32 * q;
            if (f < 6 * rows) sw[f] = in[f];
        }
        __syncwarp();
        if (lane < rows) {
            float4 x[6];
#pragma unroll
            for (int q = 0; q < 6; ++q) x[q] = sw[lane * 6 + q];
            float s = 0.0f;
#pragma unroll
            for (int q = 0; q < 6; ++q) {
                s = __fadd_rn(s, __fmul_rn(x[q].x, x[q].x));
                s = __fadd_rn(s, __fmul_rn(x[q].y, x[q].y));
                s = __fadd_rn(s, __fmul_rn(x[q].z, x[q].z));
                s = __fadd_rn(s, __fmul_rn(x[q].w, x[q].w));
            }
            s = sqrtf(s);
            if (s > 1e-8f) {
                const float inv = 1.0f / s;
#pragma unroll
                for (int q = 0; q < 6; ++q) {
                    x[q].x = __fmul_rn(x[q].x, inv);
                    x[q].y = __fmul_rn(x[q].y, inv);
                    x[q].z = __fmul_rn(x[q].z, inv);
                    x[q].w = __fmul_rn(x[q].w, inv);
                }
            }
#pragma unroll
            for (int q = 0; q < 6; ++q) sw[lane * 6 + q] = x[q];
        }
        __syncwarp();
#pragma unroll
        for (int q = 0; q < 6; ++q) {
            const int f = lane + 32 * q;
            if (f < 6 * rows) out[f] = sw[f];
        }
        __syncwarp();  // the next task's loads overwrite the stage
    }
}

// ------------------------------------------------------------------ argmax
constexpr int kTI = 128;  // rows per CTA tile
constexpr int kTJ = 128;  // columns per j-tile
constexpr int kKC = 32;   // k chunk held in shared memory
constexpr int kPitch = 128 + 4;
#ifndef M3R_ARGMAX_UNROLL
#define M3R_ARGMAX_UNROLL 2
#endif
constexpr int kArgmaxUnroll = M3R_ARGMAX_UNROLL;

// Thread (tr, tc) of a 16 x 16 grid owns rows tr*8 .. +8 and columns
// {tc*4 .. +4} U {64 + tc*4 .. +4} of the 128 x 128 tile.  Warp w holds
// tr in [4*(w/2), +4), tc in [8*(w%2), +8): lane = tr_l * 8 + tc_l.
template <int DFIX>
__global__ void __launch_bounds__(256, 2)
    argmax_kernel(const float* __restrict__ A, const float* __restrict__ B, const float* __restrict__ C1,
                  const float* __restrict__ C2, long long row0, long long row1, long long n2, int dyn_d, int n_seg,
                  unsigned long long* __restrict__ rowkey, unsigned long long* __restrict__ colkey) {
    const int D = DFIX > 0 ? DFIX : dyn_d;
    __shared__ __align__(16) float sA[kKC][kPitch];
    __shared__ __align__(16) float sB[kKC][kPitch];
    __shared__ unsigned long long sCol[4][kTJ];
    __shared__ unsigned long long sRow[2][kTI];

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int tr = 4 * (warp >> 1) + (lane >> 3);
    const int tc = 8 * (warp & 1) + (lane & 7);
    const long long i0 = row0 + static_cast<long long>(blockIdx.x) * kTI;
    const int seg = blockIdx.y;
    const long long jt_per_seg = ((n2 + kTJ - 1) / kTJ + n_seg - 1) / n_seg;
    const long long jt_begin = seg * jt_per_seg;
    long long jt_end = jt_begin + jt_per_seg;
    const long long jt_total = (n2 + kTJ - 1) / kTJ;
    if (jt_end > jt_total) jt_end = jt_total;

    float rbest[8];
    uint32_t ridx[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
        rbest[r] = -INFINITY;
        ridx[r] = 0xFFFFFFFFu;
    }

    const bool a_resident = D <= kKC;
    // rows of this thread that exist (fixed for the CTA)
    bool rv[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) rv[r] = i0 + tr * 8 + r < row1;
    // confidence weighting (matching.cpp:110-119): sim * (conf_1[i] * conf_2[j]); the
    // row confidences of this thread's 8 rows stay in registers
    const bool weighted = C1 != nullptr && C2 != nullptr;
    float cr[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
        const long long gi = i0 + tr * 8 + r;
        cr[r] = (weighted && gi < row1) ? C1[gi] : 1.0f;
    }
    for (long long jt = jt_begin; jt < jt_end; ++jt) {
        const long long j0 = jt * kTJ;
        // s[r][c]: similarity of row tr*8 + r and column (c < 4 ? tc*4 + c : 64 + tc*4 + c - 4)
        float s[8][8];
#pragma unroll
        for (int r = 0; r < 8; ++r)
#pragma unroll
            for (int c = 0; c < 8; ++c) s[r][c] = 0.0f;

        for (int kc = 0; kc < D; kc += kKC) {
            const int kn = D - kc < kKC ? D - kc : kKC;
            __syncthreads();
            // consecutive threads read consecutive floats of a row (row-major [n, D]), so
            // a warp's loads are coalesced; the chunk is stored transposed ([k][row])
            if (!a_resident || jt == jt_begin) {
                for (int e = tid; e < kTI * kn; e += 256) {
                    const int rr = e / kn, k = e - rr * kn;
                    const long long gi = i0 + rr;
                    sA[k][rr] = gi < row1 ? A[gi * D + kc + k] : 0.0f;
                }
            }
            if (DFIX > 0 && DFIX <= kKC && DFIX % 4 == 0) {
                // whole 16-byte pieces of the rows (rows are D * 4 bytes, 16-byte aligned)
                constexpr int kQ = DFIX / 4;
                for (int e = tid; e < kTJ * kQ; e += 256) {
                    const int cc = e / kQ, q = e - cc * kQ;
                    const long long gj = j0 + cc;
                    const float4 v = gj < n2 ? *reinterpret_cast<const float4*>(B + gj * D + 4 * q)
                                             : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    sB[4 * q][cc] = v.x;
                    sB[4 * q + 1][cc] = v.y;
                    sB[4 * q + 2][cc] = v.z;
                    sB[4 * q + 3][cc] = v.w;
                }
            } else {
                for (int e = tid; e < kTJ * kn; e += 256) {
                    const int cc = e / kn, k = e - cc * kn;
                    const long long gj = j0 + cc;
                    sB[k][cc] = gj < n2 ? B[gj * D + kc + k] : 0.0f;
                }
            }
            __syncthreads();
            const int KN = DFIX > 0 ? (DFIX < kKC ? DFIX : kKC) : kKC;
            // a partial unroll keeps the loop body inside the instruction cache (a full
            // unroll of 24 steps of 128 multiply / add instructions stalled on fetch)
#pragma unroll kArgmaxUnroll
            for (int k = 0; k < KN; ++k) {
                if (DFIX == 0 && k >= kn) break;
                const float4 a0 = *reinterpret_cast<const float4*>(&sA[k][tr * 8]);
                const float4 a1 = *reinterpret_cast<const float4*>(&sA[k][tr * 8 + 4]);
                const float4 b0 = *reinterpret_cast<const float4*>(&sB[k][tc * 4]);
                const float4 b1 = *reinterpret_cast<const float4*>(&sB[k][64 + tc * 4]);
                const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
                const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
                for (int r = 0; r < 8; ++r)
#pragma unroll
                    for (int c = 0; c < 8; ++c) s[r][c] = __fadd_rn(s[r][c], __fmul_rn(av[r], bv[c]));
            }
        }

        // columns of this thread that exist in this tile (32-bit offsets within the tile)
        const long long jleft = n2 - j0;
        bool cv[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) cv[c] = (c < 4 ? tc * 4 + c : 64 + tc * 4 + c - 4) < jleft;
        if (weighted) {
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const long long j = j0 + (c < 4 ? tc * 4 + c : 64 + tc * 4 + c - 4);
                const float cc = cv[c] ? C2[j] : 1.0f;
#pragma unroll
                for (int r = 0; r < 8; ++r) s[r][c] = __fmul_rn(s[r][c], __fmul_rn(cr[r], cc));
            }
        }

        // The row / column arg-max below runs in two instantiations: kEdge for the tiles
        // that hold a seed (column 0 or row 0) or ragged rows / columns, and a
        // predicate-free one for every interior tile (the condition is uniform per CTA).
        unsigned long long ck[8];
        auto argmax_tile = [&](auto edge_tag) {
            constexpr bool kEdge = decltype(edge_tag)::value;
            // ---- rows: first (lowest j) maximum over this thread's columns, in increasing j.
            // The reference seeds every row with column 0 and replaces it only on a strictly
            // greater value (matching.cpp:128-139), so column 0 is taken even when it is NaN
            // or -inf; a NaN seed is never replaced (its key, all ones, is the largest).
            // this thread holds column 0 (first tile of segment 0)
            const bool seed_col0 = kEdge && j0 == 0 && tc == 0;
#pragma unroll
            for (int r = 0; r < 8; ++r) {
                if constexpr (!kEdge) {
                    // interior tile: the row's running best rarely improves, so take the
                    // maximum (fmaxf ignores NaN, as the strict comparison does) and look for
                    // its first column only when it beats the running best
                    const float m = fmaxf(fmaxf(fmaxf(s[r][0], s[r][1]), fmaxf(s[r][2], s[r][3])),
                                          fmaxf(fmaxf(s[r][4], s[r][5]), fmaxf(s[r][6], s[r][7])));
                    if (m > rbest[r]) {
                        // first column equal to the maximum, and its own bits (-0 vs +0)
                        int mc = 7;
                        float mv = s[r][7];
#pragma unroll
                        for (int c = 6; c >= 0; --c) {
                            const bool eq = s[r][c] == m;
                            mc = eq ? c : mc;
                            mv = eq ? s[r][c] : mv;
                        }
                        rbest[r] = mv;
                        ridx[r] = static_cast<uint32_t>(j0 + (mc < 4 ? tc * 4 + mc : 64 + tc * 4 + mc - 4));
                    }
                    continue;
                }
                float m = -INFINITY;
                int mc = -1;
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    if (c == 0 && seed_col0) {
                        m = s[r][0];
                        mc = 0;
                    } else if ((!kEdge || cv[c]) && s[r][c] > m) {
                        m = s[r][c];
                        mc = c;
                    }
                }
                if (mc >= 0 && (seed_col0 || m > rbest[r])) {
                    rbest[r] = m;
                    ridx[r] = static_cast<uint32_t>(j0 + (mc < 4 ? tc * 4 + mc : 64 + tc * 4 + mc - 4));
                }
            }

            // ---- columns: first (lowest i) maximum over this thread's rows, keyed; row 0
            // seeds every column as in matching.cpp:144-155
            const bool seed_row0 = kEdge && i0 == 0 && tr == 0;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                float m = -INFINITY;
                int mr = -1;
#pragma unroll
                for (int r = 0; r < 8; ++r) {
                    if (r == 0 && seed_row0) {
                        m = s[0][c];
                        mr = 0;
                    } else if ((!kEdge || rv[r]) && s[r][c] > m) {
                        m = s[r][c];
                        mr = r;
                    }
                }
                ck[c] = mr >= 0 ? make_key(m, static_cast<uint32_t>(i0 + tr * 8 + mr)) : 0ull;
                // reduce over the 4 row groups of this warp (lanes differing in bits 3, 4)
#pragma unroll
                for (int o = 8; o <= 16; o <<= 1) {
                    const unsigned long long other = __shfl_xor_sync(0xffffffffu, ck[c], o);
                    ck[c] = other > ck[c] ? other : ck[c];
                }
            }
        };
        if (j0 == 0 || i0 == 0 || jleft < kTJ || i0 + kTI > row1)
            argmax_tile(std::true_type{});
        else
            argmax_tile(std::false_type{});
        if ((lane >> 3) == 0) {
#pragma unroll
            for (int c = 0; c < 8; ++c) sCol[warp >> 1][c < 4 ? tc * 4 + c : 64 + tc * 4 + c - 4] = ck[c];
        }
        __syncthreads();
        if (tid < kTJ) {
            unsigned long long k = sCol[0][tid];
#pragma unroll
            for (int w = 1; w < 4; ++w) k = sCol[w][tid] > k ? sCol[w][tid] : k;
            if (j0 + tid < n2 && k != 0ull) atomicMax(colkey + j0 + tid, k);
        }
    }

    // ---- row keys: reduce over the 8 column groups of the warp (lane bits 0..2), then the 2 warps
#pragma unroll
    for (int r = 0; r < 8; ++r) {
        unsigned long long k = ridx[r] != 0xFFFFFFFFu ? make_key(rbest[r], ridx[r]) : 0ull;
#pragma unroll
        for (int o = 1; o <= 4; o <<= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, k, o);
            k = other > k ? other : k;
        }
        if ((lane & 7) == 0) sRow[warp & 1][tr * 8 + r] = k;
    }
    __syncthreads();
    if (tid < kTI) {
        const unsigned long long k = sRow[0][tid] > sRow[1][tid] ? sRow[0][tid] : sRow[1][tid];
        if (i0 + tid < row1 && k != 0ull) atomicMax(rowkey + (i0 + tid - row0), k);
    }
}

// ------------------------------------------------------------------ candidates
// flag(i) = reciprocal test and threshold; per-block counts, then ordered scatter.
__device__ __forceinline__ bool cand_flag(const unsigned long long* rowkey, const unsigned long long* colkey,
                                          long long i_local, long long row0, int reciprocal, float thr,
                                          uint32_t& j_out, float& v_out) {
    const unsigned long long rk = rowkey[i_local];
    if (rk == 0ull) return false;
    const uint32_t j = 0xFFFFFFFFu - static_cast<uint32_t>(rk & 0xFFFFFFFFu);
    const float v = from_orderable(static_cast<uint32_t>(rk >> 32));
    j_out = j;
    v_out = v;
    if (reciprocal) {
        const unsigned long long ck = colkey[j];
        const long long i21 = 0xFFFFFFFFu - static_cast<uint32_t>(ck & 0xFFFFFFFFu);
        if (i21 != row0 + i_local) return false;
    }
    return v >= thr;
}

constexpr int kCandBlock = 1024;

__global__ void cand_count_kernel(const unsigned long long* __restrict__ rowkey,
                                  const unsigned long long* __restrict__ colkey, long long nrows, long long row0,
                                  int reciprocal, float thr, int* __restrict__ block_counts) {
    __shared__ int s_cnt;
    if (threadIdx.x == 0) s_cnt = 0;
    __syncthreads();
    const long long i = static_cast<long long>(blockIdx.x) * kCandBlock + threadIdx.x;
    uint32_t j;
    float v;
    const bool f = i < nrows && cand_flag(rowkey, colkey, i, row0, reciprocal, thr, j, v);
    const unsigned bal = __ballot_sync(0xffffffffu, f);
    if ((threadIdx.x & 31) == 0 && bal) atomicAdd(&s_cnt, __popc(bal));
    __syncthreads();
    if (threadIdx.x == 0) block_counts[blockIdx.x] = s_cnt;
}

__global__ void scan_counts_kernel(int* __restrict__ counts, int n, int* __restrict__ total) {
    // single block: exclusive scan in place
    __shared__ int s_carry;
    if (threadIdx.x == 0) s_carry = 0;
    __syncthreads();
    for (int base = 0; base < n; base += blockDim.x) {
        const int i = base + threadIdx.x;
        const int v = i < n ? counts[i] : 0;
        // inclusive scan within the block
        __shared__ int tmp[1024];
        tmp[threadIdx.x] = v;
        __syncthreads();
        for (int o = 1; o < blockDim.x; o <<= 1) {
            const int t = threadIdx.x >= o ? tmp[threadIdx.x - o] : 0;
            __syncthreads();
            tmp[threadIdx.x] += t;
            __syncthreads();
        }
        if (i < n) counts[i] = s_carry + tmp[threadIdx.x] - v;
        __syncthreads();
        if (threadIdx.x == blockDim.x - 1) s_carry += tmp[threadIdx.x];
        __syncthreads();
    }
    if (threadIdx.x == 0) *total = s_carry;
}

__global__ void cand_scatter_kernel(const unsigned long long* __restrict__ rowkey,
                                    const unsigned long long* __restrict__ colkey, long long nrows, long long row0,
                                    int reciprocal, float thr, const int* __restrict__ block_offsets,
                                    unsigned long long* __restrict__ ckey, uint32_t* __restrict__ cj) {
    __shared__ int s_warp[kCandBlock / 32];
    const long long i = static_cast<long long>(blockIdx.x) * kCandBlock + threadIdx.x;
    uint32_t j = 0;
    float v = 0.0f;
    const bool f = i < nrows && cand_flag(rowkey, colkey, i, row0, reciprocal, thr, j, v);
    const unsigned bal = __ballot_sync(0xffffffffu, f);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (lane == 0) s_warp[w] = __popc(bal);
    __syncthreads();
    if (threadIdx.x == 0) {
        int acc = 0;
        for (int k = 0; k < kCandBlock / 32; ++k) {
            const int t = s_warp[k];
            s_warp[k] = acc;
            acc += t;
        }
    }
    __syncthreads();
    if (f) {
        const int pos = block_offsets[blockIdx.x] + s_warp[w] + __popc(bal & ((1u << lane) - 1u));
        ckey[pos] = make_key(v, static_cast<uint32_t>(row0 + i));
        cj[pos] = j;
    }
}

// ------------------------------------------------------------------ top-k (radix select + sort)
__global__ void radix_hist_kernel(const unsigned long long* __restrict__ keys, int n, int shift,
                                  const unsigned long long* __restrict__ state, int prefix_bits,
                                  unsigned* __restrict__ hist) {
    const unsigned long long prefix = state[0];
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const unsigned long long k = keys[i];
        if (prefix_bits > 0 && (k >> (64 - prefix_bits)) != prefix) continue;
        atomicAdd(hist + ((k >> shift) & 0xFFFFull), 1u);
    }
}

// One block of kPickThreads threads: finds the digit bucket that holds the
// remaining-th largest key (buckets scanned from the highest digit down), appends
// the digit to the prefix, and clears the histogram for the next pass.
// state[0] = prefix of the digits chosen so far, state[1] = rank still to find.
constexpr int kPickThreads = 1024;
constexpr int kBinsPerThread = 65536 / kPickThreads;

__global__ void __launch_bounds__(kPickThreads) radix_pick_kernel(unsigned* __restrict__ hist,
                                                                  unsigned long long* __restrict__ state) {
    __shared__ unsigned long long s_warp[kPickThreads / 32];
    __shared__ int s_found;
    const int t = threadIdx.x, lane = t & 31, w = t >> 5;
    // thread t owns bins [hi - kBinsPerThread, hi), hi = 65536 - t * kBinsPerThread: thread 0 the highest
    const int hi = 65536 - t * kBinsPerThread;
    unsigned local = 0;
    for (int b = hi - 1; b >= hi - kBinsPerThread; --b) local += hist[b];
    // exclusive prefix over threads (descending digits): warp scan, then over warps
    unsigned long long incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) s_warp[w] = incl;
    if (t == 0) s_found = 0;
    __syncthreads();
    if (w == 0) {
        unsigned long long v = s_warp[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned long long u = __shfl_up_sync(0xffffffffu, v, o);
            if (lane >= o) v += u;
        }
        s_warp[lane] = v;  // inclusive prefix of warp sums
    }
    __syncthreads();
    const unsigned long long before = (w > 0 ? s_warp[w - 1] : 0ull) + incl - local;  // keys in higher bins
    const unsigned long long remaining = state[1];
    if (before < remaining && remaining <= before + local) {
        // the remaining-th key lies in this thread's bins
        unsigned long long cum = before;
        int b = hi - 1;
        for (; b > hi - kBinsPerThread; --b) {
            if (cum + hist[b] >= remaining) break;
            cum += hist[b];
        }
        state[0] = (state[0] << 16) | static_cast<unsigned long long>(b);
        state[1] = remaining - cum;
        s_found = 1;
    }
    __syncthreads();
    if (t == 0 && !s_found) {  // fewer keys than `remaining` (not reached when total > top_k): lowest digit
        state[0] = state[0] << 16;
        state[1] = 1;
    }
    for (int b = hi - kBinsPerThread; b < hi; ++b) hist[b] = 0;
}

__global__ void select_ge_kernel(const unsigned long long* __restrict__ keys, const uint32_t* __restrict__ cj,
                                 int n, const unsigned long long* __restrict__ kth,
                                 unsigned long long* __restrict__ out_key, uint32_t* __restrict__ out_j,
                                 int* __restrict__ counter) {
    const unsigned long long t = kth[0];
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        if (keys[i] >= t) {
            const int pos = atomicAdd(counter, 1);
            out_key[pos] = keys[i];
            out_j[pos] = cj[i];
        }
    }
}

// single block bitonic sort, descending by key, n <= 4096 (padded to a power of two)
__global__ void sort_desc_kernel(unsigned long long* __restrict__ key, uint32_t* __restrict__ val, int n) {
    __shared__ unsigned long long sk[4096];
    __shared__ uint32_t sv[4096];
    int m = 1;
    while (m < n) m <<= 1;
    for (int i = threadIdx.x; i < m; i += blockDim.x) {
        sk[i] = i < n ? key[i] : 0ull;
        sv[i] = i < n ? val[i] : 0u;
    }
    __syncthreads();
    for (int size = 2; size <= m; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < m; i += blockDim.x) {
                const int partner = i ^ stride;
                if (partner > i) {
                    const bool desc = (i & size) == 0;
                    const bool swap = desc ? (sk[i] < sk[partner]) : (sk[i] > sk[partner]);
                    if (swap) {
                        const unsigned long long tk = sk[i];
                        sk[i] = sk[partner];
                        sk[partner] = tk;
                        const uint32_t tv = sv[i];
                        sv[i] = sv[partner];
                        sv[partner] = tv;
                    }
                }
            }
            __syncthreads();
        }
    }
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        key[i] = sk[i];
        val[i] = sv[i];
    }
}

// Global-memory bitonic sort step (descending) for top_k > 4096: n is a power of two,
// one launch per (size, stride) pair.
__global__ void bitonic_step_kernel(unsigned long long* __restrict__ key, uint32_t* __restrict__ val, int n, int size,
                                    int stride) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int partner = i ^ stride;
        if (partner <= i) continue;
        const bool desc = (i & size) == 0;
        const unsigned long long a = key[i], b = key[partner];
        if (desc ? (a < b) : (a > b)) {
            key[i] = b;
            key[partner] = a;
            const uint32_t t = val[i];
            val[i] = val[partner];
            val[partner] = t;
        }
    }
}

__global__ void fill_keys_kernel(unsigned long long* __restrict__ key, uint32_t* __restrict__ val, int from, int to) {
    for (int i = from + blockIdx.x * blockDim.x + threadIdx.x; i < to; i += gridDim.x * blockDim.x) {
        key[i] = 0ull;
        val[i] = 0u;
    }
}

__global__ void finalize_kernel(const unsigned long long* __restrict__ key, const uint32_t* __restrict__ cj, int n,
                                long long* __restrict__ idx1, long long* __restrict__ idx2,
                                float* __restrict__ conf) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const unsigned long long k = key[i];
        idx1[i] = static_cast<long long>(0xFFFFFFFFu - static_cast<uint32_t>(k & 0xFFFFFFFFu));
        idx2[i] = static_cast<long long>(cj[i]);
        conf[i] = from_orderable(static_cast<uint32_t>(k >> 32));
    }
}

__global__ void decode_keys_kernel(const unsigned long long* __restrict__ key, long long n, int32_t* __restrict__ idx) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        idx[i] = static_cast<int32_t>(0xFFFFFFFFu - static_cast<uint32_t>(key[i] & 0xFFFFFFFFu));
}

int blocks_for(long long n, int b) {
    long long g = (n + b - 1) / b;
    if (g > 148LL * 16) g = 148LL * 16;
    return static_cast<int>(g < 1 ? 1 : g);
}

}  // namespace

MatchWorkspace::~MatchWorkspace() { release(); }

void MatchWorkspace::release() {
    for (void** p : {reinterpret_cast<void**>(&a), reinterpret_cast<void**>(&b), reinterpret_cast<void**>(&rowkey),
                     reinterpret_cast<void**>(&colkey), reinterpret_cast<void**>(&counts),
                     reinterpret_cast<void**>(&ckey), reinterpret_cast<void**>(&cj),
                     reinterpret_cast<void**>(&hist), reinterpret_cast<void**>(&state),
                     reinterpret_cast<void**>(&skey), reinterpret_cast<void**>(&sj), reinterpret_cast<void**>(&misc),
                     reinterpret_cast<void**>(&idx1), reinterpret_cast<void**>(&idx2),
                     reinterpret_cast<void**>(&conf), reinterpret_cast<void**>(&c1),
                     reinterpret_cast<void**>(&c2)}) {
        if (*p) cudaFree(*p);
        *p = nullptr;
    }
    cap_n = 0;
    cap_d = 0;
}

void MatchWorkspace::reserve(long long n, int d) {
    if (n <= cap_n && d <= cap_d) return;
    release();
    const long long nn = n > 0 ? n : 1;
    const int dd = d > 0 ? d : 1;
    M3R_CUDA(cudaMalloc(&a, sizeof(float) * nn * dd));
    M3R_CUDA(cudaMalloc(&b, sizeof(float) * nn * dd));
    M3R_CUDA(cudaMalloc(&rowkey, sizeof(unsigned long long) * nn));
    M3R_CUDA(cudaMalloc(&colkey, sizeof(unsigned long long) * nn));
    M3R_CUDA(cudaMalloc(&counts, sizeof(int) * ((nn + kCandBlock - 1) / kCandBlock + 1)));
    M3R_CUDA(cudaMalloc(&ckey, sizeof(unsigned long long) * nn));
    M3R_CUDA(cudaMalloc(&cj, sizeof(uint32_t) * nn));
    M3R_CUDA(cudaMalloc(&hist, sizeof(unsigned) * 65536));
    M3R_CUDA(cudaMalloc(&state, sizeof(unsigned long long) * 2));
    // selected keys: room for a power-of-two bitonic sort of up to n entries
    long long sel = 4096;
    while (sel < nn) sel <<= 1;
    M3R_CUDA(cudaMalloc(&skey, sizeof(unsigned long long) * sel));
    M3R_CUDA(cudaMalloc(&sj, sizeof(uint32_t) * sel));
    M3R_CUDA(cudaMalloc(&misc, sizeof(int) * 4));
    M3R_CUDA(cudaMalloc(&idx1, sizeof(long long) * nn));
    M3R_CUDA(cudaMalloc(&idx2, sizeof(long long) * nn));
    M3R_CUDA(cudaMalloc(&conf, sizeof(float) * nn));
    M3R_CUDA(cudaMalloc(&c1, sizeof(float) * nn));
    M3R_CUDA(cudaMalloc(&c2, sizeof(float) * nn));
    M3R_CUDA(cudaMemset(hist, 0, sizeof(unsigned) * 65536));
    cap_n = n;
    cap_d = d;
}

void match_normalize(cudaStream_t s, const float* in, float* out, long long n, int d) {
    if (n == 0) return;
    const bool aligned = (reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) % 16 == 0;
    if (d == 24 && aligned)
        normalize24_kernel<<<blocks_for(n, 256), 256, 0, s>>>(reinterpret_cast<const float4*>(in),
                                                               reinterpret_cast<float4*>(out), n);
    else
        normalize_kernel<<<blocks_for(n, 256), 256, 0, s>>>(in, out, n, d);
    M3R_CUDA(cudaGetLastError());
}

void match_normalize2(cudaStream_t s, const float* in1, float* out1, long long n1, const float* in2, float* out2,
                      long long n2, int d) {
    const bool aligned =
        ((reinterpret_cast<uintptr_t>(in1) | reinterpret_cast<uintptr_t>(out1) | reinterpret_cast<uintptr_t>(in2) |
          reinterpret_cast<uintptr_t>(out2)) %
         16) == 0;
    if (d != 24 || !aligned || n1 == 0 || n2 == 0) {
        match_normalize(s, in1, out1, n1, d);
        match_normalize(s, in2, out2, n2, d);
        return;
    }
    long long blocks = ((n1 + 31) / 32 + (n2 + 31) / 32 + kNormWarps - 1) / kNormWarps;
    if (blocks > 148LL * 8) blocks = 148LL * 8;
    normalize24_pair_kernel<<<static_cast<int>(blocks), kNormWarps * 32, 0, s>>>(
        reinterpret_cast<const float4*>(in1), reinterpret_cast<float4*>(out1), n1, reinterpret_cast<const float4*>(in2),
        reinterpret_cast<float4*>(out2), n2);
    M3R_CUDA(cudaGetLastError());
}

void match_argmax(cudaStream_t s, const float* a_norm, const float* b_norm, long long row0, long long row1,
                  long long n2, int d, unsigned long long* rowkey, unsigned long long* colkey, bool clear_colkey,
                  const float* conf_1, const float* conf_2) {
    const long long nrows = row1 - row0;
    if (nrows > 0) M3R_CUDA(cudaMemsetAsync(rowkey, 0, sizeof(unsigned long long) * nrows, s));
    if (clear_colkey && n2 > 0) M3R_CUDA(cudaMemsetAsync(colkey, 0, sizeof(unsigned long long) * n2, s));
    if (nrows <= 0 || n2 <= 0) return;
    const long long row_blocks = (nrows + kTI - 1) / kTI;
    const long long jt_total = (n2 + kTJ - 1) / kTJ;
    // column segments: enough CTAs for ~8 waves of 2 CTAs per SM
    long long seg = (148LL * 2 * 8 + row_blocks - 1) / row_blocks;
    if (seg > jt_total) seg = jt_total;
    if (seg < 1) seg = 1;
    if (seg > 65535) seg = 65535;
    M3R_REQUIRE(row_blocks <= 0x7FFFFFFFLL, "match: too many rows");
    dim3 grid(static_cast<unsigned>(row_blocks), static_cast<unsigned>(seg));
    if (d == 24)
        argmax_kernel<24><<<grid, 256, 0, s>>>(a_norm, b_norm, conf_1, conf_2, row0, row1, n2, d,
                                               static_cast<int>(seg), rowkey, colkey);
    else
        argmax_kernel<0><<<grid, 256, 0, s>>>(a_norm, b_norm, conf_1, conf_2, row0, row1, n2, d, static_cast<int>(seg),
                                              rowkey, colkey);
    M3R_CUDA(cudaGetLastError());
}

int match_select(cudaStream_t s, MatchWorkspace& ws, long long nrows, long long row0, int reciprocal, float thr,
                 int top_k, int* total_out) {
    if (total_out) *total_out = 0;
    if (nrows <= 0) return 0;
    const int nblk = static_cast<int>((nrows + kCandBlock - 1) / kCandBlock);
    int* total_d = ws.misc;
    cand_count_kernel<<<nblk, kCandBlock, 0, s>>>(ws.rowkey, ws.colkey, nrows, row0, reciprocal, thr, ws.counts);
    scan_counts_kernel<<<1, 1024, 0, s>>>(ws.counts, nblk, total_d);
    cand_scatter_kernel<<<nblk, kCandBlock, 0, s>>>(ws.rowkey, ws.colkey, nrows, row0, reciprocal, thr, ws.counts,
                                                    ws.ckey, ws.cj);
    M3R_CUDA(cudaGetLastError());
    int total = 0;
    M3R_CUDA(cudaMemcpyAsync(&total, total_d, sizeof(int), cudaMemcpyDeviceToHost, s));
    M3R_CUDA(cudaStreamSynchronize(s));
    if (total_out) *total_out = total;
    int m = total;
    if (total > top_k) {
        unsigned long long st[2] = {0ull, static_cast<unsigned long long>(top_k)};
        M3R_CUDA(cudaMemcpyAsync(ws.state, st, sizeof(st), cudaMemcpyHostToDevice, s));
        for (int pass = 0; pass < 4; ++pass) {
            radix_hist_kernel<<<blocks_for(total, 256), 256, 0, s>>>(ws.ckey, total, 48 - 16 * pass, ws.state,
                                                                      16 * pass, ws.hist);
            radix_pick_kernel<<<1, kPickThreads, 0, s>>>(ws.hist, ws.state);
        }
        M3R_CUDA(cudaMemsetAsync(ws.misc + 1, 0, sizeof(int), s));
        select_ge_kernel<<<blocks_for(total, 256), 256, 0, s>>>(ws.ckey, ws.cj, total, ws.state, ws.skey, ws.sj,
                                                                 ws.misc + 1);
        if (top_k <= 4096) {
            sort_desc_kernel<<<1, 1024, 0, s>>>(ws.skey, ws.sj, top_k);
        } else {
            int m2 = 1;
            while (m2 < top_k) m2 <<= 1;
            fill_keys_kernel<<<blocks_for(m2 - top_k, 256), 256, 0, s>>>(ws.skey, ws.sj, top_k, m2);
            for (int size = 2; size <= m2; size <<= 1)
                for (int stride = size >> 1; stride > 0; stride >>= 1)
                    bitonic_step_kernel<<<blocks_for(m2, 256), 256, 0, s>>>(ws.skey, ws.sj, m2, size, stride);
        }
        finalize_kernel<<<blocks_for(top_k, 256), 256, 0, s>>>(ws.skey, ws.sj, top_k, ws.idx1, ws.idx2, ws.conf);
        m = top_k;
    } else if (total > 0) {
        finalize_kernel<<<blocks_for(total, 256), 256, 0, s>>>(ws.ckey, ws.cj, total, ws.idx1, ws.idx2, ws.conf);
    }
    M3R_CUDA(cudaGetLastError());
    return m;
}

void match_decode(cudaStream_t s, const unsigned long long* keys, long long n, int32_t* idx) {
    if (n <= 0) return;
    decode_keys_kernel<<<blocks_for(n, 256), 256, 0, s>>>(keys, n, idx);
    M3R_CUDA(cudaGetLastError());
}

}  // namespace m3r
