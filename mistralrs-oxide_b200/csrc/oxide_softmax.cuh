// oxide_softmax.cuh -- softmax arguments and per-row helpers shared by the
// softmax kernels.
#pragma once

#include "oxide_common.cuh"

namespace oxide {

struct SmaxArgs {
    uint64_t rows;
    uint32_t cols;
    float scale;
    const float* mask;  // additive mask, indexed j % mask_len (nullable)
    uint32_t mask_len;
    FastDiv mask_div;
    const int32_t* lens;  // valid length per group of rows (nullable)
    uint64_t rows_per_len;
    uint64_t causal_q;  // 0 = no causal mask
    FastDiv len_div;     // division by rows_per_len (rows < 2^32)
    FastDiv causal_div;  // division by causal_q (rows < 2^32)
    bool narrow;         // rows < 2^32: row indices fit the 32-bit fast division
    int tpr;             // threads per row (per CTA when cl > 1)
    int cl;              // CTAs per row (cluster size)
};

// Valid key count of a row: cols, lowered by lens and by the causal mask.
// Runs for every row in every thread, so the row index is divided with the
// precomputed 32-bit multiply-shift division, not a 64-bit divide routine.
__device__ __forceinline__ uint32_t valid_len(const SmaxArgs& p, uint64_t row) {
    uint32_t len = p.cols;
    if (p.lens) {
        const uint64_t g = p.narrow ? p.len_div.div((uint32_t)row) : row / p.rows_per_len;
        const int32_t l = p.lens[g];
        const uint32_t lu = l < 0 ? 0u : (uint32_t)l;
        if (lu < len) len = lu;
    }
    if (p.causal_q) {
        const uint64_t q = p.narrow ? p.causal_div.mod((uint32_t)row) : row % p.causal_q;
        const uint64_t lim = q + 1 + (p.cols - p.causal_q);
        if (lim < len) len = (uint32_t)lim;
    }
    return len;
}

// s = x * scale, then + mask[j % mask_len] (src/ops/attention.rs:60,66-68),
// with the mask added as fma(x, scale, mask) and the exp argument s - m formed
// without a mask as fma(x, scale, -m): the same roundings as the vector
// kernels (k_softmax.cu, score_t / diff_t).
__device__ __forceinline__ float score(const SmaxArgs& p, float x, uint32_t j) {
    return p.mask ? __fmaf_rn(x, p.scale, __ldg(p.mask + p.mask_div.mod(j))) : fmul(x, p.scale);
}
__device__ __forceinline__ float score_diff(const SmaxArgs& p, float x, uint32_t j, float m) {
    return p.mask ? fsub(score(p, x, j), m) : __fmaf_rn(x, p.scale, -m);
}

}  // namespace oxide
