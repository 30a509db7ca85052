/*
 * ORACLE (test infrastructure only) -- CPU restatement of the reference's
 * reciprocal matcher, csrc/cpu/matching.cpp (Aedelon/mast3r-runtime).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
 * load this library, and only as the checker.  The product path never does.
 *
 * Arithmetic follows the reference exactly (it is built without FMA: the
 * reference CMake passes no -march, so x86-64 baseline SSE2 has no fused
 * multiply-add, and GCC does not reassociate without -ffast-math):
 *   normalize   matching.cpp:22-44   sequential  s = s + x*x  (mul, then add,
 *                                    each rounded), n = sqrtf(s),
 *                                    if n > 1e-8f: x = x * (1.0f / n)
 *   similarity  matching.cpp:53-70   sequential  d = d + a[k]*b[k], k = 0..D-1
 *   nn_12       matching.cpp:128-139 first j with the row maximum (strict >)
 *   nn_21       matching.cpp:144-155 first i with the column maximum
 *   collect     matching.cpp:161-186 i ascending; reciprocal test, sim >= thr
 *   top-k       matching.cpp:189-213 conf descending; ties (unspecified in the
 *                                    reference's partial_sort) by idx_1 ascending
 *   pts2d       matching.cpp:216-222 (idx % W, idx / W) as float
 *   confidence  matching.cpp:110-119 (when conf_1 and conf_2 are given) every
 *   weighting   similarity becomes sim * (conf_1[i] * conf_2[j]), the product
 *               of the two confidences rounded first
 *   pts3d       matching.py:144-152 (the numpy path; the C++ path leaves zeros):
 *               pts3d_1[idx_1], pts3d_2[idx_2] when pts3d maps are given
 * Unlike the reference this never materialises the N1 x N2 similarity matrix
 * (154.6 GB at N = 196,608): rows are processed in blocks and the column
 * maxima are merged across threads in row order, which gives the same
 * lowest-index tie rule.
 *
 * Build: see oracle/Makefile (-O3 -fopenmp -ffp-contract=off).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* matching.cpp:22-44 */
void oracle_normalize(float* desc, int64_t n, int d) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        float* row = desc + i * d;
        float s = 0.0f;
        for (int k = 0; k < d; ++k) {
            float p = row[k] * row[k];
            s = s + p;
        }
        s = sqrtf(s);
        if (s > 1e-8f) {
            const float inv = 1.0f / s;
            for (int k = 0; k < d; ++k) row[k] = row[k] * inv;
        }
    }
}

#define JB 256

/*
 * Row and column arg-max of sim = A . B^T over normalised inputs.
 * nn12[i] = lowest j with the maximum of row i, best12[i] that maximum;
 * nn21[j] = lowest i with the maximum of column j, best21[j] that maximum.
 * Rows [row0, row1) only (for sharded baselines); columns always all of B.
 */
void oracle_argmax_w(const float* a, const float* b, const float* c1, const float* c2, int64_t n1, int64_t n2,
                     int d, int64_t row0, int64_t row1,
                     int32_t* nn12, float* best12, int32_t* nn21, float* best21) {
    int nt = 1;
#ifdef _OPENMP
    nt = omp_get_max_threads();
#endif
    if (row1 > n1) row1 = n1;
    if (row0 < 0) row0 = 0;
    float* cbest = (float*)malloc(sizeof(float) * (size_t)(n2 > 0 ? n2 : 1) * nt);
    int32_t* cidx = (int32_t*)malloc(sizeof(int32_t) * (size_t)(n2 > 0 ? n2 : 1) * nt);
    int* touched = (int*)calloc((size_t)nt, sizeof(int));

#pragma omp parallel num_threads(nt)
    {
        int t = 0;
#ifdef _OPENMP
        t = omp_get_thread_num();
#endif
        const int64_t span = row1 - row0;
        const int64_t r0 = row0 + span * t / nt;
        const int64_t r1 = row0 + span * (t + 1) / nt;
        float* cb = cbest + (size_t)n2 * t;
        int32_t* ci = cidx + (size_t)n2 * t;
        float* bt = (float*)malloc(sizeof(float) * (size_t)JB * (d > 0 ? d : 1));
        float dot[JB];
        if (r1 > r0) touched[t] = 1;
        for (int64_t j = 0; j < n2; ++j) { cb[j] = 0.0f; ci[j] = -1; }
        for (int64_t i = r0; i < r1; ++i) { nn12[i] = 0; best12[i] = 0.0f; }
        for (int64_t j0 = 0; j0 < n2; j0 += JB) {
            const int jn = (int)((n2 - j0) < JB ? (n2 - j0) : JB);
            /* B block transposed to [k][jj] so the jj loop vectorises; the
             * per-element operation sequence is unchanged. */
            for (int jj = 0; jj < jn; ++jj)
                for (int k = 0; k < d; ++k) bt[(size_t)k * JB + jj] = b[(j0 + jj) * d + k];
            for (int64_t i = r0; i < r1; ++i) {
                const float* ar = a + i * d;
                for (int jj = 0; jj < jn; ++jj) dot[jj] = 0.0f;
                for (int k = 0; k < d; ++k) {
                    const float ak = ar[k];
                    const float* br = bt + (size_t)k * JB;
                    for (int jj = 0; jj < jn; ++jj) {
                        float p = ak * br[jj];
                        dot[jj] = dot[jj] + p;
                    }
                }
                if (c1 && c2) {
                    const float ci = c1[i];
                    for (int jj = 0; jj < jn; ++jj) {
                        const float w = ci * c2[j0 + jj];
                        dot[jj] = dot[jj] * w;
                    }
                }
                float best = best12[i];
                int32_t bj = nn12[i];
                int jstart = 0;
                if (j0 == 0) { best = dot[0]; bj = 0; jstart = 1; }
                for (int jj = jstart; jj < jn; ++jj)
                    if (dot[jj] > best) { best = dot[jj]; bj = (int32_t)(j0 + jj); }
                best12[i] = best;
                nn12[i] = bj;
                /* matching.cpp:144-155 seeds every column with row 0 and replaces it
                 * only on a strictly greater value: a thread's partial starts at the
                 * global row 0 or at its first non-NaN value (a NaN elsewhere never wins) */
                for (int jj = 0; jj < jn; ++jj) {
                    const int64_t j = j0 + jj;
                    if ((ci[j] < 0 && (i == 0 || dot[jj] == dot[jj])) || (ci[j] >= 0 && dot[jj] > cb[j])) {
                        cb[j] = dot[jj];
                        ci[j] = (int32_t)i;
                    }
                }
            }
        }
        free(bt);
    }
    /* merge thread partials in row order: strict > keeps the lowest i */
#pragma omp parallel for schedule(static)
    for (int64_t j = 0; j < n2; ++j) {
        float best = 0.0f;
        int32_t bi = -1;
        for (int t = 0; t < nt; ++t) {
            if (!touched[t]) continue;
            const float v = cbest[(size_t)n2 * t + j];
            const int32_t ii = cidx[(size_t)n2 * t + j];
            if (ii < 0) continue;
            if (bi < 0 || v > best) { best = v; bi = ii; }
        }
        nn21[j] = bi < 0 ? 0 : bi;
        best21[j] = best;
    }
    free(cbest);
    free(cidx);
    free(touched);
}

void oracle_argmax(const float* a, const float* b, int64_t n1, int64_t n2, int d,
                   int64_t row0, int64_t row1,
                   int32_t* nn12, float* best12, int32_t* nn21, float* best21) {
    oracle_argmax_w(a, b, NULL, NULL, n1, n2, d, row0, row1, nn12, best12, nn21, best21);
}

typedef struct { float c; int64_t i; int64_t j; } cand_t;

static int cand_cmp(const void* x, const void* y) {
    const cand_t* p = (const cand_t*)x;
    const cand_t* q = (const cand_t*)y;
    if (p->c > q->c) return -1;
    if (p->c < q->c) return 1;
    return (p->i < q->i) ? -1 : (p->i > q->i);
}

/*
 * Full reciprocal_match (matching.cpp:85-237) on raw descriptors d1 [n, d],
 * d2 [n, d] of an H x W map (n = H * W).  Outputs are sized top_k (or n when
 * top_k >= n).  Returns the number of matches written, or -1 on bad input.
 */
int64_t oracle_match_w(const float* d1, const float* d2, const float* c1, const float* c2,
                       const float* p3_1, const float* p3_2, int64_t n, int d, int width,
                       int top_k, int reciprocal, float thr,
                       int64_t* idx1, int64_t* idx2, float* conf, float* pts2d_1, float* pts2d_2,
                       float* pts3d_1, float* pts3d_2, int32_t* nn12_out, int32_t* nn21_out) {
    if (n < 0 || d <= 0 || top_k < 0 || (n > 0 && width <= 0)) return -1;
    if (n == 0) return 0;
    float* a = (float*)malloc(sizeof(float) * (size_t)n * d);
    float* b = (float*)malloc(sizeof(float) * (size_t)n * d);
    memcpy(a, d1, sizeof(float) * (size_t)n * d);
    memcpy(b, d2, sizeof(float) * (size_t)n * d);
    oracle_normalize(a, n, d);
    oracle_normalize(b, n, d);
    int32_t* nn12 = (int32_t*)malloc(sizeof(int32_t) * (size_t)n);
    int32_t* nn21 = (int32_t*)malloc(sizeof(int32_t) * (size_t)n);
    float* b12 = (float*)malloc(sizeof(float) * (size_t)n);
    float* b21 = (float*)malloc(sizeof(float) * (size_t)n);
    oracle_argmax_w(a, b, c1, c2, n, n, d, 0, n, nn12, b12, nn21, b21);
    cand_t* cand = (cand_t*)malloc(sizeof(cand_t) * (size_t)n);
    int64_t m = 0;
    for (int64_t i = 0; i < n; ++i) {
        const int64_t j = nn12[i];
        if (reciprocal && nn21[j] != i) continue;
        const float s = b12[i]; /* == sim[i][nn12[i]] */
        if (s >= thr) { cand[m].c = s; cand[m].i = i; cand[m].j = j; ++m; }
    }
    if (m > top_k) {
        qsort(cand, (size_t)m, sizeof(cand_t), cand_cmp);
        m = top_k;
    }
    for (int64_t k = 0; k < m; ++k) {
        idx1[k] = cand[k].i;
        idx2[k] = cand[k].j;
        conf[k] = cand[k].c;
        pts2d_1[2 * k + 0] = (float)(cand[k].i % width);
        pts2d_1[2 * k + 1] = (float)(cand[k].i / width);
        pts2d_2[2 * k + 0] = (float)(cand[k].j % width);
        pts2d_2[2 * k + 1] = (float)(cand[k].j / width);
        for (int q = 0; q < 3; ++q) {
            if (pts3d_1) pts3d_1[3 * k + q] = p3_1 ? p3_1[3 * cand[k].i + q] : 0.0f;
            if (pts3d_2) pts3d_2[3 * k + q] = p3_2 ? p3_2[3 * cand[k].j + q] : 0.0f;
        }
    }
    if (nn12_out) memcpy(nn12_out, nn12, sizeof(int32_t) * (size_t)n);
    if (nn21_out) memcpy(nn21_out, nn21, sizeof(int32_t) * (size_t)n);
    free(a); free(b); free(nn12); free(nn21); free(b12); free(b21); free(cand);
    return m;
}

int64_t oracle_match(const float* d1, const float* d2, int64_t n, int d, int width,
                     int top_k, int reciprocal, float thr,
                     int64_t* idx1, int64_t* idx2, float* conf, float* pts2d_1, float* pts2d_2,
                     int32_t* nn12_out, int32_t* nn21_out) {
    return oracle_match_w(d1, d2, NULL, NULL, NULL, NULL, n, d, width, top_k, reciprocal, thr, idx1, idx2, conf,
                          pts2d_1, pts2d_2, NULL, NULL, nn12_out, nn21_out);
}

/*
 * Isolated non-causal attention for one (sequence, head) slice, fp32:
 * O = softmax(Q K^T * scale) V, scores materialised, as the reference's
 * csrc/cpu/attention.cpp:118-159 (multi_head_attention) computes per head.
 * Used as the CPU baseline of the attention kernel; parity of the kernel is
 * checked against a float64 restatement in the tests.
 */
void oracle_attention_head(const float* q, const float* k, const float* v, float* o,
                           int nq, int nk, int dh, float scale, float* scratch /* nk floats */) {
    for (int i = 0; i < nq; ++i) {
        float mx = -INFINITY;
        for (int j = 0; j < nk; ++j) {
            float s = 0.0f;
            for (int t = 0; t < dh; ++t) s += q[i * dh + t] * k[j * dh + t];
            s *= scale;
            scratch[j] = s;
            if (s > mx) mx = s;
        }
        float sum = 0.0f;
        for (int j = 0; j < nk; ++j) { scratch[j] = expf(scratch[j] - mx); sum += scratch[j]; }
        const float inv = 1.0f / sum;
        for (int t = 0; t < dh; ++t) o[i * dh + t] = 0.0f;
        for (int j = 0; j < nk; ++j) {
            const float p = scratch[j] * inv;
            for (int t = 0; t < dh; ++t) o[i * dh + t] += p * v[j * dh + t];
        }
    }
}

void oracle_attention(const float* q, const float* k, const float* v, float* o,
                      int64_t n_slices, int nq, int nk, int dh, float scale) {
#pragma omp parallel
    {
        float* scratch = (float*)malloc(sizeof(float) * (size_t)(nk > 0 ? nk : 1));
#pragma omp for schedule(dynamic, 1)
        for (int64_t s = 0; s < n_slices; ++s)
            oracle_attention_head(q + s * nq * dh, k + s * nk * dh, v + s * nk * dh,
                                  o + s * nq * dh, nq, nk, dh, scale, scratch);
        free(scratch);
    }
}
