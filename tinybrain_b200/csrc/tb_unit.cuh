// tb_unit.cuh -- step bookkeeping shared by the LM-head epilogues of the
// per-op GEMV kernel (tb_gemv.cu) and the persistent decode-step kernels
// (tb_step.cu, tb_flow.cu): the argmax key and the per-sequence advance.
#pragma once

#include "tb_common.cuh"

namespace tb {

// Step bookkeeping of one sequence after its LM head (ModelRunner.swift:251-292):
// the argmax becomes the next input once the prompt is consumed (and is
// recorded as a generated token); before that the next prompt token is fed.
__device__ __forceinline__ void finish_sequence_step(SeqState& sq, int m, int* out_tokens, const int* prompt,
                                                     int prompt_stride) {
    const unsigned long long b = atomicAdd(&sq.best, 0ull);
    const int tok = (int)(0xFFFFFFFFu - (uint32_t)(b & 0xFFFFFFFFull));
    int next;
    if (sq.pos >= sq.n_prompt - 1) {
        if (sq.n_out < sq.max_out) out_tokens[(size_t)m * sq.max_out + sq.n_out] = tok;
        sq.n_out += 1;
        next = tok;
    } else {
        next = prompt[(size_t)m * prompt_stride + sq.pos + 1];
    }
    sq.token = next;
    sq.pos += 1;
    sq.best = 0ull;
}

// Packed argmax key: larger value first; among equal values the lower index
// (Sampler.swift:126-138).
__device__ __forceinline__ unsigned long long argmax_key(float v, int n) {
    return ((unsigned long long)float_order_key(v) << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)n);
}

}  // namespace tb
