// oxide_rowstream.cuh -- declarations shared by the row kernels: softmax
// arguments and their per-row helpers, and the launchers of the streaming
// (bulk-copy pipelined) row kernels defined in k_rowstream.cu.
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
__device__ __host__ __forceinline__ uint32_t valid_len_of(uint64_t cols, const int32_t* lens_val,
                                                          uint64_t causal_q, uint64_t row) {
    uint64_t len = cols;
    if (lens_val) {
        int64_t l = *lens_val;
        if (l < 0) l = 0;
        if ((uint64_t)l < len) len = (uint64_t)l;
    }
    if (causal_q) {
        uint64_t lim = row % causal_q + 1 + (cols - causal_q);
        if (lim < len) len = lim;
    }
    return (uint32_t)len;
}

__device__ __forceinline__ uint32_t valid_len(const SmaxArgs& p, uint64_t row) {
    return valid_len_of(p.cols, p.lens ? p.lens + row / p.rows_per_len : nullptr, p.causal_q, row);
}

// s = x * scale, then + mask[j % mask_len]: src/ops/attention.rs:60,66-68.
__device__ __forceinline__ float score(const SmaxArgs& p, float x, uint32_t j) {
    float s = fmul(x, p.scale);
    if (p.mask) s = fadd(s, __ldg(p.mask + p.mask_div.mod(j)));
    return s;
}

// Streaming launchers: return true if the shape was eligible and a kernel was
// enqueued, false if the caller must use another kernel.
template <typename T>
bool rms_stream_launch(const T* x, const T* r, const T* w, T* h, T* y, uint64_t rows,
                       uint32_t cols, float eps, cudaStream_t st);
template <typename T>
bool smax_stream_launch(const T* x, T* out, const SmaxArgs& p, cudaStream_t st);

}  // namespace oxide
