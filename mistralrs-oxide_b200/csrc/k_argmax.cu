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

// Few long rows (decode logits), vector path: a cluster of CTAs per row.
// Each CTA scans its slice keeping (best value, index) and the first index
// that holds a number (not NaN), reduces both over the CTA, and thread 0
// stores them into rank 0's shared memory (distributed shared memory); after
// one cluster barrier (release / acquire) rank 0 merges the CTAs' pairs and
// writes the row's index -- the first non-NaN index when the maximum is -inf
// (0 if every element is NaN), as in argmax_kernel.  One cluster barrier per
// row and no second scan; the slots are double-buffered by row parity, so a
// CTA already on the next row cannot overwrite a pair rank 0 has not read.
template <typename T>
__global__ void __launch_bounds__(256)
    argmax_cluster_kernel(const T* x, uint64_t rows, uint32_t cols, uint32_t* idx) {
    pdl_begin();
    constexpr int V = Vec<T>::N;
    constexpr int UNROLL = 8;
    __shared__ Best red[8];
    __shared__ uint32_t redn[8];
    __shared__ Best slots[2][8];
    __shared__ uint32_t nslots[2][8];
    cg::cluster_group cluster = cg::this_cluster();
    const uint32_t cl = cluster.num_blocks(), rank = cluster.block_rank();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t n = cols / V, per = (n + cl - 1) / cl;
    const uint32_t lo = min(n, rank * per), hi = min(n, lo + per);
    Best* slot0 = cluster.map_shared_rank(&slots[0][0], 0);
    uint32_t* nslot0 = cluster.map_shared_rank(&nslots[0][0], 0);
    uint32_t par = 0;
    for (uint64_t row = blockIdx.x / cl; row < rows; row += gridDim.x / cl, par ^= 1u) {
        const T* xr = x + row * cols;
        float bv = -INFINITY;
        uint32_t bi = NONE, nn = NONE;
        for (uint32_t u0 = lo + threadIdx.x; u0 < hi; u0 += blockDim.x * UNROLL) {
            uint4 raw[UNROLL];
#pragma unroll
            for (int k = 0; k < UNROLL; ++k) {
                const uint32_t u = u0 + k * blockDim.x;
                if (u < hi) raw[k] = ld_stream(xr + (uint64_t)u * V);
            }
#pragma unroll
            for (int k = 0; k < UNROLL; ++k) {
                const uint32_t u = u0 + k * blockDim.x;
                if (u < hi) {
                    float f[V];
                    Vec<T>::unpack(raw[k], f);
#pragma unroll
                    for (int e = 0; e < V; ++e) {
                        if (f[e] > bv) {
                            bv = f[e];
                            bi = u * V + e;
                        }
                        if (nn == NONE && f[e] == f[e]) nn = u * V + e;  // the thread scans in index order
                    }
                }
            }
        }
        const Best b = warp_best(Best{bv, bi});
        const uint32_t m = __reduce_min_sync(0xffffffffu, nn);
        if (lane == 0) {
            red[warp] = b;
            redn[warp] = m;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            Best r = red[0];
            uint32_t mm = redn[0];
            for (int w = 1; w < (int)(blockDim.x >> 5); ++w) {
                r = better(r, red[w]);
                mm = min(mm, redn[w]);
            }
            slot0[par * 8 + rank] = r;
            nslot0[par * 8 + rank] = mm;
        }
        cluster.sync();  // rank 0 sees every CTA's pair; red[] may be written again
        if (rank == 0 && threadIdx.x == 0) {
            Best r = slots[par][0];
            uint32_t mm = nslots[par][0];
            for (uint32_t q = 1; q < cl; ++q) {
                r = better(r, slots[par][q]);
                mm = min(mm, nslots[par][q]);
            }
            idx[row] = r.i != NONE ? r.i : (mm == NONE ? 0u : mm);
        }
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
    cudaError_t e = vec && cl > 1 ? cudaLaunchKernelEx(&cfg, argmax_cluster_kernel<T>, x, rows, c32, idx)
                    : vec         ? cudaLaunchKernelEx(&cfg, argmax_kernel<T, true>, x, rows, c32, idx, cl)
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
