// Reciprocal matcher building blocks (matcher.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace m3r {

// Device buffers for one matcher call of up to cap_n descriptors per set.
struct MatchWorkspace {
    float* a = nullptr;               // normalised set A [n, d]
    float* b = nullptr;               // normalised set B [n, d]
    unsigned long long* rowkey = nullptr;
    unsigned long long* colkey = nullptr;
    int* counts = nullptr;
    unsigned long long* ckey = nullptr;
    uint32_t* cj = nullptr;
    unsigned* hist = nullptr;
    unsigned long long* state = nullptr;
    unsigned long long* skey = nullptr;
    uint32_t* sj = nullptr;
    int* misc = nullptr;
    long long* idx1 = nullptr;
    long long* idx2 = nullptr;
    float* conf = nullptr;
    float* c1 = nullptr;              // confidence maps (weighted matching)
    float* c2 = nullptr;
    long long cap_n = 0;
    int cap_d = 0;

    ~MatchWorkspace();
    void reserve(long long n, int d);
    void release();
};

// Reference normalisation (csrc/cpu/matching.cpp:22-44), out may alias in.
void match_normalize(cudaStream_t s, const float* in, float* out, long long n, int d);
// Both sets in one launch where the layout allows (d == 24, 16-byte aligned), else two.
void match_normalize2(cudaStream_t s, const float* in1, float* out1, long long n1, const float* in2, float* out2,
                      long long n2, int d);

// Row keys of rows [row0, row1) of A (rowkey[i - row0]) and column keys of all n2
// columns of B (colkey[j], merged with atomicMax; cleared first when asked).  With
// conf_1 (indexed by global row) and conf_2 (by column) both given, every similarity
// is weighted by conf_1[i] * conf_2[j] (csrc/cpu/matching.cpp:110-119).
void match_argmax(cudaStream_t s, const float* a_norm, const float* b_norm, long long row0, long long row1,
                  long long n2, int d, unsigned long long* rowkey, unsigned long long* colkey, bool clear_colkey,
                  const float* conf_1 = nullptr, const float* conf_2 = nullptr);

// Reciprocal / threshold / top-k over rows [row0, row0 + nrows) with keys in ws;
// results in ws.idx1 / ws.idx2 / ws.conf.  Returns the match count (<= top_k);
// *total_out (optional) gets the number of candidates before the top-k cut.
int match_select(cudaStream_t s, MatchWorkspace& ws, long long nrows, long long row0, int reciprocal, float thr,
                 int top_k, int* total_out = nullptr);

// Index part of keys -> int32 (nn_12 / nn_21 for tests).
void match_decode(cudaStream_t s, const unsigned long long* keys, long long n, int32_t* idx);

}  // namespace m3r
