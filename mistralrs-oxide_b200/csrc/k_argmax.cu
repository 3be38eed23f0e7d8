// k_argmax.cu -- per-row argmax (greedy next-token selection over logits).
//
// API addition: the reference's only argmax-like path is sample_top_k with
// k = 1 after a stable descending sort (src/tokenizer.rs:213-232): it returns
// the lowest index among equal maxima.  This kernel reproduces that choice,
// with +0 == -0 and NaN ranked below every number.
//
// Design: every element becomes one 64-bit key
//     (order-preserving 32-bit image of the value) << 32 | (0xffffffff - index)
// so "largest value, then lowest index" is a plain unsigned max, reduced with
// shuffles and shared memory.  Many rows: one CTA per row.  Few long rows
// (decode logits): a cluster of CTAs splits each row and combines the CTA
// keys through distributed shared memory.
#include <cooperative_groups.h>

#include "oxide_common.cuh"

namespace cg = cooperative_groups;

namespace oxide {

__device__ __forceinline__ uint64_t amax_key(float v, uint32_t j) {
    uint32_t k;
    if (v != v) {
        k = 0u;  // NaN: below -inf
    } else {
        if (v == 0.0f) v = 0.0f;  // -0 ranks equal to +0
        const uint32_t u = __float_as_uint(v);
        k = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    }
    return ((uint64_t)k << 32) | (uint64_t)(0xffffffffu - j);
}

template <typename T, bool VEC>
__global__ void __launch_bounds__(256)
    argmax_kernel(const T* x, uint64_t rows, uint32_t cols, uint32_t* idx, int cl) {
    constexpr int V = VEC ? Vec<T>::N : 1;
    constexpr int UNROLL = 4;
    __shared__ uint64_t red[8];
    __shared__ uint64_t slot;
    const uint32_t n = cols / V;  // units (vectors or elements) per row
    int rank = 0;
    if (cl > 1) rank = (int)cg::this_cluster().block_rank();
    const uint32_t per = (n + cl - 1) / cl;
    const uint32_t lo = rank * per, hi = min(n, lo + per);
    for (uint64_t row = blockIdx.x / cl; row < rows; row += gridDim.x / cl) {
        const T* xr = x + row * cols;
        uint64_t best = 0;
        for (uint32_t u0 = lo + threadIdx.x; u0 < hi; u0 += blockDim.x * UNROLL) {
            if (VEC) {
                uint4 raw[UNROLL];
#pragma unroll
                for (int k = 0; k < UNROLL; ++k) {
                    const uint32_t u = u0 + k * blockDim.x;
                    if (u < hi) raw[k] = ld_stream(xr + (uint64_t)u * Vec<T>::N);
                }
#pragma unroll
                for (int k = 0; k < UNROLL; ++k) {
                    const uint32_t u = u0 + k * blockDim.x;
                    if (u < hi) {
                        float f[Vec<T>::N];
                        Vec<T>::unpack(raw[k], f);
#pragma unroll
                        for (int e = 0; e < Vec<T>::N; ++e) {
                            const uint64_t key = amax_key(f[e], u * Vec<T>::N + e);
                            best = key > best ? key : best;
                        }
                    }
                }
            } else {
#pragma unroll
                for (int k = 0; k < UNROLL; ++k) {
                    const uint32_t u = u0 + k * blockDim.x;
                    if (u < hi) {
                        const uint64_t key = amax_key(Vec<T>::load1(xr + u), u);
                        best = key > best ? key : best;
                    }
                }
            }
        }
        best = group_reduce(best, red, (int)blockDim.x, OpMaxU64());
        if (cl > 1) {
            cg::cluster_group cluster = cg::this_cluster();
            if (threadIdx.x == 0) slot = best;
            cluster.sync();
            if (rank == 0 && threadIdx.x == 0) {
                uint64_t b = 0;
                for (int q = 0; q < cl; ++q) {
                    const uint64_t v = *cluster.map_shared_rank(&slot, q);
                    b = v > b ? v : b;
                }
                best = b;
            }
            cluster.sync();  // peers' slots stay valid until rank 0 has read them
        }
        if (rank == 0 && threadIdx.x == 0)
            idx[row] = 0xffffffffu - (uint32_t)(best & 0xffffffffu);
    }
}

template <typename T>
static int argmax_entry(const char* name, const T* x, uint64_t rows, uint64_t cols,
                        uint32_t* idx, cudaStream_t st) {
    OXIDE_INJECT(name);
    if (rows == 0) return OXIDE_OK;
    OXIDE_REQUIRE(x && idx, name, "null pointer");
    OXIDE_REQUIRE(cols >= 1 && cols < 0xffffffffull, name, "cols must be in [1, 2^32 - 1)");
    OXIDE_REQUIRE(rows <= UINT64_MAX / cols, name, "rows * cols overflows");
    constexpr int V = Vec<T>::N;
    const bool vec = cols % V == 0 && aligned16(x);
    const uint64_t units = vec ? cols / V : cols;
    // Split a row over a cluster when there are too few rows to fill the GPU
    // and each CTA would still get at least 4 units per thread.
    int cl = 1;
    const uint64_t target = 2ull * sm_count();
    while (cl < 8 && rows * cl < target && units / (2 * cl) >= 256 * 4) cl *= 2;
    const uint64_t cap = ((uint64_t)1 << 30) / cl;
    const uint64_t groups = rows < cap ? rows : cap;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(groups * cl), 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const uint32_t c32 = (uint32_t)cols;
    cudaError_t e = vec ? cudaLaunchKernelEx(&cfg, argmax_kernel<T, true>, x, rows, c32, idx, cl)
                        : cudaLaunchKernelEx(&cfg, argmax_kernel<T, false>, x, rows, c32, idx, cl);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return set_error(OXIDE_ERR_LAUNCH, "%s: launch failed: %s", name, cudaGetErrorString(e));
    }
    return check_launch(name);
}

}  // namespace oxide

using oxide::bf16_t;

extern "C" {

int oxide_argmax_rows_f32(const float* x, uint64_t rows, uint64_t cols, uint32_t* idx,
                          oxide_stream_t stream) {
    return oxide::argmax_entry<float>("oxide_argmax_rows_f32", x, rows, cols, idx, stream);
}
int oxide_argmax_rows_bf16(const oxide_bf16* x, uint64_t rows, uint64_t cols, uint32_t* idx,
                           oxide_stream_t stream) {
    return oxide::argmax_entry<bf16_t>("oxide_argmax_rows_bf16", x, rows, cols, idx, stream);
}

}  // extern "C"
