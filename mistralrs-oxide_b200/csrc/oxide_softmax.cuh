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
    int tpr;            // threads per row (per CTA when cl > 1)
    int cl;             // CTAs per row (cluster size)
};

// Valid key count of a row: cols, lowered by lens and by the causal mask.
__device__ __forceinline__ uint32_t valid_len(const SmaxArgs& p, uint64_t row) {
    uint64_t len = p.cols;
    if (p.lens) {
        int64_t l = p.lens[row / p.rows_per_len];
        if (l < 0) l = 0;
        if ((uint64_t)l < len) len = (uint64_t)l;
    }
    if (p.causal_q) {
        uint64_t lim = row % p.causal_q + 1 + (p.cols - p.causal_q);
        if (lim < len) len = lim;
    }
    return (uint32_t)len;
}

// s = x * scale, then + mask[j % mask_len]: src/ops/attention.rs:60,66-68.
__device__ __forceinline__ float score(const SmaxArgs& p, float x, uint32_t j) {
    float s = fmul(x, p.scale);
    if (p.mask) s = fadd(s, __ldg(p.mask + p.mask_div.mod(j)));
    return s;
}

}  // namespace oxide
