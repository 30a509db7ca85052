#pragma once

#include <cuda_runtime.h>

#include "tmap.h"

namespace m3r {

// O[seq, tok, head*64] = softmax(Q K^T * scale) V per (seq, head); Q [seq, head, nq, 64],
// K/V [seq, head, nk, 64], all 16-bit of type `dt` (Dt).  Query sequence s attends to
// key/value sequence s.  err: device status word that a timed-out wait sets (may be null).
void attention_fwd(cudaStream_t s, int dt, const void* q, const void* k, const void* v, void* out, int n_seq,
                   int heads, int nq, int nk, float scale, int* err);

}  // namespace m3r
