// k_softmax.cu -- softmax(x, dim) and scale + mask + softmax over rows.
//
// Reference: src/ops/activation.rs:95-120 (max, exp(x - max) with a running
// sum, divide) and the scale/mask/softmax block of scaled_dot_product_attention
// (src/ops/attention.rs:41,60,63-79: s = dot * scale; s += mask[j % len];
// softmax over the key axis).
//
// Design (rows of a contiguous [rows, cols] tensor):
//   * a row is owned by `tpr` threads of one CTA (a warp for rows of up to
//     256 vectors, several rows per CTA) or, for long decode rows, by a
//     thread-block cluster of `cl` CTAs that exchange the row max and the row
//     sum through distributed shared memory;
//   * the row is read once into registers with 16-byte streaming loads,
//     max/sum are reduced with fixed trees (deterministic), and the
//     probabilities are written once;
//   * keys at or beyond a row's valid length (lens / causal) are written as 0
//     and never read.
// softmax over an inner (non-last) dim, odd lengths, unaligned pointers and
// rows beyond the register budget take multi-pass kernels.
#include <cooperative_groups.h>

#include "oxide_rowstream.cuh"

namespace cg = cooperative_groups;

namespace oxide {

// 16 row elements per thread run 4 CTAs of 256 threads per SM (<= 64
// registers); 32 elements per thread run 2 (<= 128 registers); the short-row
// warp instances (< 16 elements) run 3, whose unrolled exp/divide sequences
// need a little more than 64 registers.
template <typename T, int VPT>
constexpr int smax_min_blocks() {
    return VPT * Vec<T>::N == 16 ? 4 : (VPT * Vec<T>::N < 16 ? 3 : 2);
}

template <typename T, int VPT>
__global__ void __launch_bounds__(256, smax_min_blocks<T, VPT>())
    smax_rows_kernel(const T* x, T* out, SmaxArgs p) {
    constexpr int V = Vec<T>::N;
    __shared__ float red[8];
    __shared__ float cl_slot[2];
    const uint32_t nvec = p.cols / V;
    int rank = 0, rpc = 1, sub = 0, t = threadIdx.x;
    uint64_t row_first, row_step;
    uint32_t vlo = 0, vhi = nvec;
    if (p.cl > 1) {
        rank = (int)cg::this_cluster().block_rank();
        const uint32_t per = (nvec + p.cl - 1) / p.cl;
        vlo = rank * per;
        vhi = min(nvec, vlo + per);
        row_first = blockIdx.x / p.cl;
        row_step = gridDim.x / p.cl;
    } else {
        rpc = blockDim.x / p.tpr;
        sub = threadIdx.x / p.tpr;
        t = threadIdx.x % p.tpr;
        row_first = (uint64_t)blockIdx.x * rpc;
        row_step = (uint64_t)gridDim.x * rpc;
    }
    for (uint64_t row0 = row_first; row0 < p.rows; row0 += row_step) {
        const uint64_t row = row0 + sub;
        const bool active = row < p.rows;
        const uint32_t len = active ? valid_len(p, row) : 0;
        const T* xr = x + row * p.cols;
        T* orow = out + row * p.cols;
        float s[VPT][V];
        uint4 raw[VPT];
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const uint32_t j = vlo + t + k * p.tpr;
            if (active && j < vhi && j * V < len) raw[k] = ld_stream(xr + (uint64_t)j * V);
        }
        float m = -INFINITY;
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const uint32_t j = vlo + t + k * p.tpr;
            if (active && j < vhi && j * V < len) {
                Vec<T>::unpack(raw[k], s[k]);
#pragma unroll
                for (int e = 0; e < V; ++e) {
                    const uint32_t c = j * V + e;
                    s[k][e] = c < len ? score(p, s[k][e], c) : -INFINITY;
                    m = fmaxf(m, s[k][e]);
                }
            } else {
#pragma unroll
                for (int e = 0; e < V; ++e) s[k][e] = -INFINITY;
            }
        }
        m = group_reduce(m, red, p.tpr, OpMaxF());
        if (p.cl > 1) {
            cg::cluster_group cluster = cg::this_cluster();
            if (threadIdx.x == 0) cl_slot[0] = m;
            cluster.sync();
            float mm = -INFINITY;
            for (int q = 0; q < p.cl; ++q) mm = fmaxf(mm, *cluster.map_shared_rank(&cl_slot[0], q));
            m = mm;
        }
        float sum = 0.0f;
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
#pragma unroll
            for (int e = 0; e < V; ++e) {
                s[k][e] = expf(fsub(s[k][e], m));  // exp(-inf - m) = 0 for masked keys
                sum = fadd(sum, s[k][e]);
            }
        }
        sum = group_reduce(sum, red, p.tpr, OpAddF());
        if (p.cl > 1) {
            cg::cluster_group cluster = cg::this_cluster();
            if (threadIdx.x == 0) cl_slot[1] = sum;
            cluster.sync();
            float tot = 0.0f;
            for (int q = 0; q < p.cl; ++q) tot = fadd(tot, *cluster.map_shared_rank(&cl_slot[1], q));
            sum = tot;
            cluster.sync();  // peers finished reading this CTA's slots
        }
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const uint32_t j = vlo + t + k * p.tpr;
            if (active && j < vhi) {
                float o[V];
                if (j * V < len) {
#pragma unroll
                    for (int e = 0; e < V; ++e)
                        o[e] = (j * V + e < len) ? fdiv(s[k][e], sum) : 0.0f;
                } else {
#pragma unroll
                    for (int e = 0; e < V; ++e) o[e] = 0.0f;
                }
                st_stream(orow + (uint64_t)j * V, Vec<T>::pack(o));
            }
        }
    }
}

// Multi-pass row kernel: any cols, any alignment.  One CTA per row; reads the
// unmasked part of the row three times (max, sum, write).
template <typename T>
__global__ void __launch_bounds__(256) smax_rows_scalar_kernel(const T* x, T* out, SmaxArgs p) {
    __shared__ float red[8];
    for (uint64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
        const uint32_t len = valid_len(p, row);
        const T* xr = x + row * p.cols;
        T* orow = out + row * p.cols;
        float m = -INFINITY;
        for (uint32_t j = threadIdx.x; j < len; j += blockDim.x)
            m = fmaxf(m, score(p, Vec<T>::load1(xr + j), j));
        m = group_reduce(m, red, (int)blockDim.x, OpMaxF());
        float sum = 0.0f;
        for (uint32_t j = threadIdx.x; j < len; j += blockDim.x)
            sum = fadd(sum, expf(fsub(score(p, Vec<T>::load1(xr + j), j), m)));
        sum = group_reduce(sum, red, (int)blockDim.x, OpAddF());
        __syncthreads();  // every thread has read its inputs before any write (in place)
        for (uint32_t j = threadIdx.x; j < p.cols; j += blockDim.x) {
            float o = 0.0f;
            if (j < len) o = fdiv(expf(fsub(score(p, Vec<T>::load1(xr + j), j), m)), sum);
            Vec<T>::store1(orow + j, o);
        }
    }
}

// softmax over a non-last dim: x viewed as [outer, dim, inner]; one thread
// per (outer, inner) column, consecutive threads on consecutive inner indices
// (coalesced).  out must not alias x.
template <typename T>
__global__ void __launch_bounds__(256)
    smax_inner_kernel(const T* x, T* out, uint64_t outer, uint64_t dim, uint64_t inner) {
    const uint64_t total = outer * inner;
    for (uint64_t c = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; c < total;
         c += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t base = (c / inner) * dim * inner + (c % inner);
        float m = -INFINITY;
        for (uint64_t d = 0; d < dim; ++d) m = fmaxf(m, Vec<T>::load1(x + base + d * inner));
        float sum = 0.0f;
        for (uint64_t d = 0; d < dim; ++d)
            sum = fadd(sum, expf(fsub(Vec<T>::load1(x + base + d * inner), m)));
        for (uint64_t d = 0; d < dim; ++d)
            Vec<T>::store1(out + base + d * inner,
                           fdiv(expf(fsub(Vec<T>::load1(x + base + d * inner), m)), sum));
    }
}

template <typename T, int VPT>
static cudaError_t launch_rows(const T* x, T* out, SmaxArgs p, cudaStream_t st) {
    const uint64_t cap = (uint64_t)1 << 30;
    if (p.cl > 1) {
        const uint64_t clusters = p.rows < cap / p.cl ? p.rows : cap / p.cl;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)(clusters * p.cl), 1, 1);
        cfg.blockDim = dim3(p.tpr, 1, 1);
        cfg.dynamicSmemBytes = 0;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = p.cl;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, smax_rows_kernel<T, VPT>, x, out, p);
    }
    const int rpc = 256 / p.tpr;
    const uint64_t want = (p.rows + rpc - 1) / rpc;
    smax_rows_kernel<T, VPT><<<(unsigned)(want < cap ? want : cap), p.tpr * rpc, 0, st>>>(x, out, p);
    return cudaSuccess;
}

// Kernel shape for rows of nvec 16-byte vectors.  Every thread holds 16 row
// elements (32 for rows beyond 8 x 4096 elements); returns VPT (0 = the
// multi-pass fallback) and sets the threads per row and the cluster size.
template <typename T>
static int smax_shape(uint64_t nvec, SmaxArgs& p) {
    constexpr int VPT16 = 16 / Vec<T>::N;
    p.cl = 1;
    if (nvec <= 32ull * VPT16) {  // a warp per row, 8 rows per CTA
        p.tpr = 32;
        int vpt = 1;
        while ((uint64_t)vpt * 32 < nvec) vpt *= 2;
        return vpt;
    }
    if (nvec <= 256ull * VPT16) {  // 64..256 threads per row, 256 / tpr rows per CTA
        uint64_t tpr = 64;
        while (tpr * VPT16 < nvec) tpr *= 2;
        p.tpr = (int)tpr;
        return VPT16;
    }
    p.tpr = 256;  // a cluster of up to 8 CTAs x 256 threads per row (DSMEM exchange)
    int vpt = VPT16;
    uint64_t cl = (nvec + 256ull * VPT16 - 1) / (256ull * VPT16);
    if (cl > 8) {
        vpt = 2 * VPT16;
        cl = (nvec + 256ull * vpt - 1) / (256ull * vpt);
        if (cl > 8) return 0;
    }
    int c2 = 1;
    while ((uint64_t)c2 < cl) c2 *= 2;
    p.cl = c2;
    return vpt;
}

template <typename T>
static int rows_dispatch(const char* name, const T* x, T* out, SmaxArgs p, cudaStream_t st) {
    constexpr int V = Vec<T>::N;
    // Rows of 1-32 KiB stream through the shared-memory bulk-copy ring.
    if (smax_stream_launch<T>(x, out, p, st)) return check_launch(name);
    const bool vec = p.cols % V == 0 && aligned16(x) && aligned16(out);
    const int vpt = vec ? smax_shape<T>(p.cols / V, p) : 0;
    const uint64_t cap = (uint64_t)1 << 30;
    cudaError_t e = cudaSuccess;
    if (vpt == 1) e = launch_rows<T, 1>(x, out, p, st);
    else if (vpt == 2) e = launch_rows<T, 2>(x, out, p, st);
    else if (vpt == 4) e = launch_rows<T, 4>(x, out, p, st);
    else if (vpt == 8) {
        if constexpr (V == 4) e = launch_rows<T, 8>(x, out, p, st);
    } else {
        smax_rows_scalar_kernel<T><<<(unsigned)(p.rows < cap ? p.rows : cap), 256, 0, st>>>(x, out, p);
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        return set_error(OXIDE_ERR_LAUNCH, "%s: launch failed: %s", name, cudaGetErrorString(e));
    }
    return check_launch(name);
}

template <typename T>
static int scale_mask_entry(const char* name, const T* x, T* out, uint64_t rows, uint64_t cols,
                            float scale, const float* mask, uint64_t mask_len,
                            const int32_t* lens, uint64_t rows_per_len, uint64_t causal_q,
                            cudaStream_t st) {
    OXIDE_INJECT(name);
    if (rows == 0) return OXIDE_OK;
    OXIDE_REQUIRE(x && out, name, "null pointer");
    OXIDE_REQUIRE(cols >= 1 && cols < (1ull << 31), name, "cols must be in [1, 2^31)");
    OXIDE_REQUIRE(rows <= UINT64_MAX / cols, name, "rows * cols overflows");
    OXIDE_REQUIRE(!mask || (mask_len >= 1 && mask_len < (1ull << 32)), name,
                  "mask_len must be in [1, 2^32)");
    OXIDE_REQUIRE(!lens || rows_per_len >= 1, name, "rows_per_len must be >= 1 with lens");
    OXIDE_REQUIRE(causal_q <= cols, name, "causal_q_len must be <= cols");
    SmaxArgs p{};
    p.rows = rows;
    p.cols = (uint32_t)cols;
    p.scale = scale;
    p.mask = mask;
    p.mask_len = mask ? (uint32_t)mask_len : 1u;
    p.mask_div = FastDiv(p.mask_len);
    p.lens = lens;
    p.rows_per_len = lens ? rows_per_len : 1;
    p.causal_q = causal_q;
    return rows_dispatch<T>(name, x, out, p, st);
}

template <typename T>
static int softmax_entry(const char* name, const T* x, T* out, uint64_t outer, uint64_t dim,
                         uint64_t inner, cudaStream_t st) {
    OXIDE_INJECT(name);
    if (outer == 0 || inner == 0) return OXIDE_OK;
    OXIDE_REQUIRE(x && out, name, "null pointer");
    OXIDE_REQUIRE(dim >= 1 && dim < (1ull << 31), name, "dim must be in [1, 2^31)");
    OXIDE_REQUIRE(outer <= UINT64_MAX / dim / inner, name, "outer * dim * inner overflows");
    if (inner == 1) {
        SmaxArgs p{};
        p.rows = outer;
        p.cols = (uint32_t)dim;
        p.scale = 1.0f;  // x * 1.0f is exact: plain softmax
        p.mask_len = 1;
        p.mask_div = FastDiv(1);
        p.rows_per_len = 1;
        return rows_dispatch<T>(name, x, out, p, st);
    }
    OXIDE_REQUIRE(x != out, name, "out must not alias x when inner > 1");
    const uint64_t total = outer * inner;
    const uint64_t blocks = (total + 255) / 256;
    const uint64_t cap = (uint64_t)sm_count() * 8;
    smax_inner_kernel<T><<<(unsigned)(blocks < cap ? blocks : cap), 256, 0, st>>>(x, out, outer, dim,
                                                                                  inner);
    return check_launch(name);
}

}  // namespace oxide

using oxide::bf16_t;

extern "C" {

int oxide_softmax_f32(const float* x, float* out, uint64_t outer, uint64_t dim, uint64_t inner,
                      oxide_stream_t stream) {
    return oxide::softmax_entry<float>("oxide_softmax_f32", x, out, outer, dim, inner, stream);
}
int oxide_softmax_bf16(const oxide_bf16* x, oxide_bf16* out, uint64_t outer, uint64_t dim,
                       uint64_t inner, oxide_stream_t stream) {
    return oxide::softmax_entry<bf16_t>("oxide_softmax_bf16", x, out, outer, dim, inner, stream);
}
int oxide_scale_mask_softmax_f32(const float* x, float* out, uint64_t rows, uint64_t cols,
                                 float scale, const float* mask, uint64_t mask_len,
                                 const int32_t* lens, uint64_t rows_per_len,
                                 uint64_t causal_q_len, oxide_stream_t stream) {
    return oxide::scale_mask_entry<float>("oxide_scale_mask_softmax_f32", x, out, rows, cols,
                                          scale, mask, mask_len, lens, rows_per_len,
                                          causal_q_len, stream);
}
int oxide_scale_mask_softmax_bf16(const oxide_bf16* x, oxide_bf16* out, uint64_t rows,
                                  uint64_t cols, float scale, const float* mask,
                                  uint64_t mask_len, const int32_t* lens,
                                  uint64_t rows_per_len, uint64_t causal_q_len,
                                  oxide_stream_t stream) {
    return oxide::scale_mask_entry<bf16_t>("oxide_scale_mask_softmax_bf16", x, out, rows, cols,
                                           scale, mask, mask_len, lens, rows_per_len,
                                           causal_q_len, stream);
}

}  // extern "C"
