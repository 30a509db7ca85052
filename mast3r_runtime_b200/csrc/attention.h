#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "tmap.h"

namespace m3r {

// O[seq, tok, head*64] = softmax(Q K^T * scale) V per (seq, head); Q [seq, head, nq, 64],
// K/V [seq, head, nk, 64], all bf16.  Query sequence s attends to key/value sequence s.
// err: device status word that a timed-out wait sets (may be null).
void attention_fwd(cudaStream_t s, const __nv_bfloat16* q, const __nv_bfloat16* k, const __nv_bfloat16* v,
                   __nv_bfloat16* out, int n_seq, int heads, int nq, int nk, float scale, int* err);

}  // namespace m3r
