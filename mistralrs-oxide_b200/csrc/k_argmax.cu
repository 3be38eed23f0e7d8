// k_argmax.cu -- per-row argmax (greedy next-token selection over logits).
//
// API addition: the reference's only argmax-like path is sample_top_k with
// k = 1 after a stable descending sort (src/tokenizer.rs:213-232): it returns
// the lowest index among equal maxima.  This kernel reproduces that choice,
// with +0 == -0 and NaN ranked below every number.
//
// Design: each thread scans its elements in increasing index order keeping
// (best value, index) and replacing only on a strictly greater value -- three
// instructions per element, ties keep the earlier index, NaN never wins.
// Thread results merge with shuffles and shared memory (larger value, then
// lower index); few long rows (decode logits) are split over a thread-block
// cluster whose CTAs merge through distributed shared memory.  A row whose
// maximum is -inf (only -inf and NaN) finds no strictly greater element; for
// it the CTA runs a second scan for the first non-NaN index (0 if none).
#include <cooperative_groups.h>

#include "oxide_common.cuh"

namespace cg = cooperative_groups;

namespace oxide {

constexpr uint32_t NONE = 0xffffffffu;

struct Best {
    float v;
    uint32_t i;
};

__device__ __forceinline__ Best better(Best a, Best b) {
    // b wins with a larger value, or an equal value at a lower index.
    const bool take = (b.v > a.v) || (b.v == a.v && b.i < a.i);
    return take ? b : a;
}

__device__ __forceinline__ Best warp_best(Best b) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        Best c{__shfl_xor_sync(0xffffffffu, b.v, o), __shfl_xor_sync(0xffffffffu, b.i, o)};
        b = better(b, c);
    }
    return b;
}

// Block-wide best (every thread receives it).  Contains __syncthreads().
__device__ __forceinline__ Best block_best(Best b, Best* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    b = warp_best(b);
    if (lane == 0) red[warp] = b;
    __syncthreads();
    Best r = red[0];
    for (int w = 1; w < nw; ++w) r = better(r, red[w]);
    __syncthreads();
    return r;
}

__device__ __forceinline__ uint32_t block_min_u32(uint32_t v, uint32_t* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) red[warp] = v;
    __syncthreads();
    uint32_t r = red[0];
    for (int w = 1; w < nw; ++w) r = min(r, red[w]);
    __syncthreads();
    return r;
}

template <typename T, bool VEC>
__global__ void __launch_bounds__(256)
    argmax_kernel(const T* x, uint64_t rows, uint32_t cols, uint32_t* idx, int cl) {
    pdl_begin();
    constexpr int V = VEC ? Vec<T>::N : 1;
    // 8 loads in flight per thread: bf16 [131072 x 32000] 1287 -> 1216 us and f32
    // [64 x 32000] 5.24 -> 5.11 us against 4
    constexpr int UNROLL = 8;
    __shared__ Best red[8];
    __shared__ uint32_t redi[8];
    __shared__ Best slot;
    __shared__ uint32_t slot_first;
    const uint32_t n = cols / V;  // units (vectors or elements) per row
    int rank = 0;
    if (cl > 1) rank = (int)cg::this_cluster().block_rank();
    const uint32_t per = (n + cl - 1) / cl;
    const uint32_t lo = rank * per, hi = min(n, lo + per);
    for (uint64_t row = blockIdx.x / cl; row < rows; row += gridDim.x / cl) {
        const T* xr = x + row * cols;
        float bv = -INFINITY;
        uint32_t bi = NONE;
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
                            if (f[e] > bv) {
                                bv = f[e];
                                bi = u * Vec<T>::N + e;
                            }
                        }
                    }
                }
            } else {
#pragma unroll
                for (int k = 0; k < UNROLL; ++k) {
                    const uint32_t u = u0 + k * blockDim.x;
                    if (u < hi) {
                        const float f = Vec<T>::load1(xr + u);
                        if (f > bv) {
                            bv = f;
                            bi = u;
                        }
                    }
                }
            }
        }
        Best b = block_best(Best{bv, bi}, red);
        if (cl > 1) {
            cg::cluster_group cluster = cg::this_cluster();
            if (threadIdx.x == 0) slot = b;
            cluster.sync();
            Best m = *cluster.map_shared_rank(&slot, 0);
            for (int q = 1; q < cl; ++q) m = better(m, *cluster.map_shared_rank(&slot, q));
            b = m;
        }
        uint32_t result = b.i;
        if (b.i == NONE) {
            // Maximum is -inf: the first non-NaN element wins (0 if all NaN).
            // Uniform across the cluster: every CTA saw the same merged result.
            uint32_t first = NONE;
            for (uint32_t j = rank * per * V + threadIdx.x; j < min(cols, (rank * per + per) * V);
                 j += blockDim.x) {
                const float f = Vec<T>::load1(xr + j);
                if (f == f) {
                    first = j;
                    break;
                }
            }
            first = block_min_u32(first, redi);
            if (cl > 1) {
                cg::cluster_group cluster = cg::this_cluster();
                if (threadIdx.x == 0) slot_first = first;
                cluster.sync();
                for (int q = 0; q < cl; ++q) first = min(first, *cluster.map_shared_rank(&slot_first, q));
            }
            result = first == NONE ? 0u : first;
        }
        if (cl > 1) cg::this_cluster().sync();  // peers' slots stay valid until read
        if (rank == 0 && threadIdx.x == 0) idx[row] = result;
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
    // Split a row over a cluster of up to 8 CTAs while all CTAs still fit one
    // wave and each keeps at least 4 units per thread (one round of loads).
    // (One 1024-thread CTA per row instead, with no cluster barrier: 5.95 us
    // against 5.4 us at [64 x 32000] f32.)
    int cl = 1;
    const uint64_t slots = (uint64_t)resident_blocks(
        vec ? reinterpret_cast<const void*>(argmax_kernel<T, true>)
            : reinterpret_cast<const void*>(argmax_kernel<T, false>), 256, 0);
    while (cl < 8 && rows * (uint64_t)(2 * cl) <= slots && units / (2 * cl) >= 256 * 4) cl *= 2;
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
    // No programmatic-dependent-launch attribute on this cluster launch:
    // measured at [64 x 32000] f32, 5.13 us per launch without it against
    // 5.43 us with it (the kernel's griddepcontrol instructions are then no-ops).
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
