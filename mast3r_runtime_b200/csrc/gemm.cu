// Launchers and the instantiated (operand type, BN, A mode, epilogue) variants of the
// tcgen05 GEMM.
#include <cstring>
#include <mutex>
#include <string>

#include "gemm.h"

namespace m3r {

int num_sms() {
    int dev = 0, n = 0;
    M3R_CUDA(cudaGetDevice(&dev));
    M3R_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
    return n;
}

GemmParams gemm_params() {
    GemmParams p;
    std::memset(&p, 0, sizeof(p));
    p.act = ACT_NONE;
    p.desc_dim = 24;
    return p;
}

namespace {

struct Maps {
    CUtensorMap a0, a1, b;
    CUtensorMap c[3];  // epilogue TMA-store maps (unused ones zero)
};

template <class T, int BN, int AMODE, int EPI, int CG>
void launch(cudaStream_t s, const Maps& m, const GemmParams& p) {
    using C = GemmCfg<BN, CG, AMODE, epi_ring<EPI, CG>()>;
    auto kern = gemm_tc_kernel<T, BN, AMODE, EPI, CG>;
    static std::once_flag once;  // per instantiation; the attribute is set on every device
    std::call_once(once, [&] {
        int ndev = 0;
        M3R_CUDA(cudaGetDeviceCount(&ndev));
        int cur = 0;
        M3R_CUDA(cudaGetDevice(&cur));
        for (int d = 0; d < ndev; ++d) {
            M3R_CUDA(cudaSetDevice(d));
            M3R_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES));
        }
        M3R_CUDA(cudaSetDevice(cur));
    });
    const int units = ((p.tiles_m + CG - 1) / CG) * p.tiles_n;  // tiles of CG x 128 rows
    if (units == 0) return;
    const int max_units = num_sms() / CG;
    const int grid = CG * (units < max_units ? units : max_units);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = C::SMEM_BYTES;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CG;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    M3R_CUDA(cudaLaunchKernelEx(&cfg, kern, m.a0, m.a1, m.b, m.c[0], m.c[1], m.c[2], p));
}

#define M3R_GEMM_CASE(BN_, AM_, EPI_)                                \
    if (bn == BN_ && amode == AM_ && epi == EPI_) {                  \
        if (cg == 2)                                                 \
            launch<T, BN_, AM_, EPI_, 2>(s, m, p);                   \
        else                                                         \
            launch<T, BN_, AM_, EPI_, 1>(s, m, p);                   \
        return;                                                      \
    }

// A_CONV3W variants exist for CTA pairs only
#define M3R_GEMM_CASE_PAIR(BN_, AM_, EPI_)                 \
    if (bn == BN_ && amode == AM_ && epi == EPI_ && cg == 2) { \
        launch<T, BN_, AM_, EPI_, 2>(s, m, p);             \
        return;                                            \
    }

template <class T>
void dispatch_t(cudaStream_t s, int bn, int amode, int epi, int cg, const Maps& m, const GemmParams& p) {
    M3R_GEMM_CASE(256, A_PLAIN, EPI_BF16)
    M3R_GEMM_CASE(128, A_PLAIN, EPI_BF16)
    M3R_GEMM_CASE(256, A_PLAIN, EPI_F32)
    M3R_GEMM_CASE(128, A_PLAIN, EPI_F32)
    M3R_GEMM_CASE(256, A_PLAIN, EPI_F32_RESID)
    M3R_GEMM_CASE(128, A_PLAIN, EPI_F32_RESID)
    M3R_GEMM_CASE(256, A_PLAIN, EPI_F32_RESID_LK)
    M3R_GEMM_CASE(128, A_PLAIN, EPI_F32_RESID_LK)
    M3R_GEMM_CASE(256, A_PLAIN, EPI_HEADS)
    M3R_GEMM_CASE(128, A_PLAIN, EPI_HEADS)
    M3R_GEMM_CASE(192, A_PLAIN, EPI_DESC)
    M3R_GEMM_CASE(96, A_PLAIN, EPI_DESC)
    M3R_GEMM_CASE(256, A_PLAIN, EPI_CONVT)
    M3R_GEMM_CASE(256, A_CONCAT, EPI_BF16)
    M3R_GEMM_CASE(256, A_CONV3, EPI_BF16)
    M3R_GEMM_CASE(128, A_CONV3, EPI_BF16)
    M3R_GEMM_CASE(128, A_CONV3, EPI_HEAD4)
    M3R_GEMM_CASE(128, A_CONV3, EPI_F32)  // conv parity test entry
    M3R_GEMM_CASE(256, A_CONV3, EPI_F32)
    M3R_GEMM_CASE_PAIR(128, A_CONV3W, EPI_BF16)
    M3R_GEMM_CASE_PAIR(128, A_CONV3W, EPI_HEAD4)
    M3R_GEMM_CASE_PAIR(128, A_CONV3W, EPI_F32)  // conv parity test entry
    throw Error(kErrArg, "no GEMM variant for bn=" + std::to_string(bn) + " amode=" + std::to_string(amode) +
                             " epi=" + std::to_string(epi));
}

void dispatch(cudaStream_t s, int dt, int bn, int amode, int epi, int cg, const Maps& m, const GemmParams& p) {
    if (dt == DT_F16)
        dispatch_t<__half>(s, bn, amode, epi, cg, m, p);
    else if (dt == DT_BF16)
        dispatch_t<__nv_bfloat16>(s, bn, amode, epi, cg, m, p);
    else
        throw Error(kErrArg, "unknown operand type " + std::to_string(dt));
}

int cdiv(long long a, long long b) { return static_cast<int>((a + b - 1) / b); }

// CTAs per tile.  A CTA pair stages half as much B per CTA (more pipeline stages,
// half the B traffic per SM) and launches as many CTAs as single-CTA tiles would,
// so it is used whenever there are row blocks to pair.
int pick_cg(int cta_pair, int tiles_m) {
    if (cta_pair == 0) return 1;
    if (cta_pair == 1) return 2;
    return tiles_m >= 2 ? 2 : 1;
}

// Epilogue TMA maps: BF16 / F32 / F32_RESID outputs as a [rows, N] matrix (and the
// F32_RESID residual, loaded by TMA, as map 1) and EPI_HEADS sections as
// [seq * heads, n_tok, 64], with 32-row boxes.  p.c_tma stays 0 (row-staged thread
// stores) when the layout does not allow whole 32-row boxes; EPI_F32_RESID has no
// such fallback and requires 16-byte aligned rows.
void out_maps(int dt, int epi, long long rows, bool rows_consecutive, GemmParams& p, Maps& m) {
    std::memset(m.c, 0, sizeof(m.c));
    p.c_tma = 0;
    const bool out_ok = p.out != nullptr && reinterpret_cast<uintptr_t>(p.out) % 16 == 0;
    if (epi == EPI_F32_RESID) {
        M3R_REQUIRE(rows_consecutive && out_ok && (p.ldo * 4) % 16 == 0 && p.resid != nullptr &&
                        reinterpret_cast<uintptr_t>(p.resid) % 16 == 0 && (p.ldr * 4) % 16 == 0,
                    "gemm: the residual epilogue needs 16-byte aligned output and residual rows");
        m.c[0] = tmap_2d_f32(p.out, rows, p.N, p.ldo, 32);
        m.c[1] = tmap_2d_f32(p.resid, rows, p.N, p.ldr, 32);
        p.c_tma = 1;
        return;
    }
    if (!rows_consecutive) return;
    if (epi == EPI_BF16) {
        if (!out_ok || (p.ldo * 2) % 16 != 0) return;
        m.c[0] = tmap_2d(dt, p.out, rows, p.N, p.ldo, 32);
        p.c_tma = 1;
    } else if (epi == EPI_F32) {
        if (!out_ok || (p.ldo * 4) % 16 != 0) return;
        m.c[0] = tmap_2d_f32(p.out, rows, p.N, p.ldo, 32);
        p.c_tma = 1;
    } else if (epi == EPI_HEADS) {
        if (p.n_tok <= 0 || p.n_tok % 32 != 0 || rows % p.n_tok != 0 || p.sec_len % 64 != 0) return;
        const long long nseq_heads = rows / p.n_tok * (p.sec_len / 64);
        for (int i = 0; i < 3; ++i) {
            if (p.sec_out[i] == nullptr) continue;
            if (reinterpret_cast<uintptr_t>(p.sec_out[i]) % 16 != 0) return;
            m.c[i] = tmap_3d_rows64(dt, p.sec_out[i], p.n_tok, nseq_heads, 32);
        }
        p.c_tma = 1;
    }
}

}  // namespace

void gemm_rows(cudaStream_t s, int dt, int bn, int epi, const void* A, long long lda, int M, int K, const void* W,
               long long ldw, int N, GemmParams p, int cta_pair) {
    M3R_REQUIRE(M >= 0 && N > 0 && K > 0, "gemm: bad shape");
    if (M == 0) return;
    p.M = M;
    p.N = N;
    p.num_kb = cdiv(K, 64);
    p.tiles_m = cdiv(M, 128);
    p.tiles_n = cdiv(N, bn);
    const int cg = pick_cg(cta_pair, p.tiles_m);
    Maps m;
    m.a0 = m.a1 = tmap_2d(dt, A, M, K, lda, 128);
    m.b = tmap_2d(dt, W, N, K, ldw, bn / cg);
    out_maps(dt, epi, M, true, p, m);
    // residual epilogue: the long-K instantiation above 16 k-blocks (see epi_ring)
    if (epi == EPI_F32_RESID && p.num_kb > 16) epi = EPI_F32_RESID_LK;
    dispatch(s, dt, bn, A_PLAIN, epi, cg, m, p);
}

void gemm_concat(cudaStream_t s, int dt, int bn, int epi, const void* A0, long long lda0, int K0, const void* A1,
                 long long lda1, int K1, int M, const void* W, long long ldw, int N, GemmParams p, int cta_pair) {
    M3R_REQUIRE(K0 % 64 == 0, "gemm_concat: K0 must be a multiple of 64");
    if (M == 0) return;
    p.M = M;
    p.N = N;
    p.a_split_kb = K0 / 64;
    p.num_kb = K0 / 64 + cdiv(K1, 64);
    p.tiles_m = cdiv(M, 128);
    p.tiles_n = cdiv(N, bn);
    const int cg = pick_cg(cta_pair, p.tiles_m);
    Maps m;
    m.a0 = tmap_2d(dt, A0, M, K0, lda0, 128);
    m.a1 = tmap_2d(dt, A1, M, K1, lda1, 128);
    m.b = tmap_2d(dt, W, N, K0 + K1, ldw, bn / cg);
    out_maps(dt, epi, M, true, p, m);
    dispatch(s, dt, bn, A_CONCAT, epi, cg, m, p);
}

void gemm_conv3(cudaStream_t s, int dt, int bn, int epi, const void* X, int n, int h, int w, int c, int cstride,
                const void* W, int N, GemmParams p, int cta_pair) {
    M3R_REQUIRE(n > 0 && h > 0 && w > 0 && c > 0 && cstride >= c, "gemm_conv3: bad shape");
    int wbox = 1;
    while (wbox * 2 <= 128 && w % (wbox * 2) == 0) wbox *= 2;
    const int hbox = 128 / wbox;
    M3R_REQUIRE(hbox <= 256, "gemm_conv3: box too tall");
    const int cblocks = cdiv(c, 64);
    p.M = n * h * w;
    p.N = N;
    p.cv_H = h;
    p.cv_W = w;
    p.cv_cblocks = cblocks;
    p.cv_wbox = wbox;
    p.cv_hbox = hbox;
    p.cv_tx = w / wbox;
    p.cv_ty = cdiv(h, hbox);
    p.num_kb = 9 * cblocks;
    p.tiles_m = n * p.cv_tx * p.cv_ty;
    p.tiles_n = cdiv(N, bn);
    const int cg = pick_cg(cta_pair, p.tiles_m);
    // 128-pixel row tiles on CTA pairs with 128 output channels per tile: one wide box
    // per (dy, channel block) serves the three dx taps
    const bool wide = cg == 2 && wbox == 128 && bn == 128;
    if (wide) p.num_kb = 3 * cblocks;
    Maps m;
    m.a0 = m.a1 = tmap_nhwc(dt, X, n, h, w, c, cstride, hbox, wide ? GemmCfg<128, 2, A_CONV3W>::WIDE_ROWS : wbox);
    m.b = tmap_2d(dt, W, N, 9LL * cblocks * 64, 9LL * cblocks * 64, bn / cg);
    // a warp's 32 output pixels are consecutive in one image row when boxes are >= 32 wide
    out_maps(dt, epi, p.M, wbox >= 32, p, m);
    dispatch(s, dt, bn, wide ? A_CONV3W : A_CONV3, epi, cg, m, p);
}

}  // namespace m3r
