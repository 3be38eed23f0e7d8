// k_softmax.cu -- softmax(x, dim) and scale + mask + softmax over rows.
//
// Reference: src/ops/activation.rs:95-120 (max, exp(x - max) with a running
// sum, divide) and the scale/mask/softmax block of scaled_dot_product_attention
// (src/ops/attention.rs:41,60,63-79: s = dot * scale; s += mask[j % len];
// softmax over the key axis).
//
// Design (rows of a contiguous [rows, cols] tensor):
//   * rows that tile a 256-thread CTA (a warp or a power-of-two group per
//     row, 256 / group rows per CTA) read straight from HBM, many CTAs per SM
//     in flight; long rows run one CTA of up to 512 threads per row, or, when
//     there are too few rows to fill the GPU, a thread-block cluster of up to
//     8 CTAs per row that exchange the row max and sum through distributed
//     shared memory;
//   * each thread holds its part of the row PACKED (bf16 stays 2 bytes per
//     element), 32 elements for bf16 and 16 for f32; the kernels are
//     instruction-bound, so fully valid 16-byte vectors take a path without
//     per-element bounds checks and the additive mask is a template
//     parameter; max and sum use fixed reduction trees (deterministic); the
//     divide by the row sum is RowDiv (the correctly rounded quotient);
//   * keys at or beyond a row's valid length (lens / causal) are written as 0
//     and never read;
//   * bf16 rows of whole vectors up to 2048 keys without an additive mask (the
//     attention-probability shape) take a warp-per-row kernel whose f32
//     intermediate is accurate to ~1e-5 relative, far inside the one-bf16-ulp
//     output tolerance (see smax_bf16_warp_kernel).
// softmax over an inner (non-last) dim, odd lengths, unaligned pointers and
// rows beyond the register budget take multi-pass kernels.
#include <cooperative_groups.h>

#include <type_traits>

#include "oxide_softmax.cuh"

namespace cg = cooperative_groups;

namespace oxide {

// ---- per-thread row chunk: VPT packed vectors j = j0 + k * jstep ------------
template <bool MASK>
__device__ __forceinline__ float score_t(const SmaxArgs& p, float x, uint32_t c) {
    float s = fmul(x, p.scale);
    if (MASK) s = fadd(s, __ldg(p.mask + p.mask_div.mod(c)));
    return s;
}

// Scores of keys c, c + 1 on the paired f32 pipe (same roundings as score_t).
template <bool MASK>
__device__ __forceinline__ float2 score2(const SmaxArgs& p, float x0, float x1, uint32_t c) {
    float2 s = fmul2(f2(x0, x1), f2(p.scale, p.scale));
    if (MASK)
        s = fadd2(s, f2(__ldg(p.mask + p.mask_div.mod(c)), __ldg(p.mask + p.mask_div.mod(c + 1))));
    return s;
}

// Max of the valid scores of the chunk (vectors j < jhi, keys c < len).
template <typename T, int VPT, bool MASK>
__device__ __forceinline__ float chunk_max(const uint4 (&raw)[VPT], const SmaxArgs& p, uint32_t j0,
                                           uint32_t jstep, uint32_t jhi, uint32_t len) {
    constexpr int V = Vec<T>::N;
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const uint32_t j = j0 + k * jstep;
        if (j < jhi && j * V < len) {
            float f[V];
            Vec<T>::unpack(raw[k], f);
            if (j * V + V <= len) {
#pragma unroll
                for (int e = 0; e < V; e += 2) {
                    const float2 s = score2<MASK>(p, f[e], f[e + 1], j * V + e);
                    m = fmaxf(m, fmaxf(s.x, s.y));
                }
            } else {
#pragma unroll
                for (int e = 0; e < V; ++e)
                    if (j * V + e < len) m = fmaxf(m, score_t<MASK>(p, f[e], j * V + e));
            }
        }
    }
    return m;
}

// ev = exp(score - m) for valid keys (0 for masked keys of a partial vector);
// returns the thread's sum (two lane accumulators, combined at the end).
template <typename T, int VPT, bool MASK>
__device__ __forceinline__ float chunk_exp(const uint4 (&raw)[VPT], float (&ev)[VPT][Vec<T>::N],
                                           const SmaxArgs& p, uint32_t j0, uint32_t jstep,
                                           uint32_t jhi, uint32_t len, float m) {
    constexpr int V = Vec<T>::N;
    const float2 nm = f2(-m, -m);
    float2 acc = f2(0.0f, 0.0f);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const uint32_t j = j0 + k * jstep;
        if (j < jhi && j * V < len) {
            float f[V];
            Vec<T>::unpack(raw[k], f);
            if (j * V + V <= len) {  // every key valid: no per-key checks
#pragma unroll
                for (int e = 0; e < V; e += 2) {
                    const float2 d = fadd2(score2<MASK>(p, f[e], f[e + 1], j * V + e), nm);
                    ev[k][e] = expf(d.x);
                    ev[k][e + 1] = expf(d.y);
                    acc = fadd2(acc, f2(ev[k][e], ev[k][e + 1]));
                }
            } else {  // the one vector of the row that straddles len
#pragma unroll
                for (int e = 0; e < V; e += 2) {
                    const float2 d = fadd2(score2<MASK>(p, f[e], f[e + 1], j * V + e), nm);
                    ev[k][e] = j * V + e < len ? expf(d.x) : 0.0f;
                    ev[k][e + 1] = j * V + e + 1 < len ? expf(d.y) : 0.0f;
                    acc = fadd2(acc, f2(ev[k][e], ev[k][e + 1]));
                }
            }
        }
    }
    return fadd(acc.x, acc.y);
}

// Write p = ev / sum (0 beyond len) for every vector j < jhi of the chunk.
// RowDiv's paired fast path per vector; a vector holding a numerator outside
// its range (or a row whose sum is outside it) is redone with the IEEE divide.
template <typename T, int VPT>
__device__ __forceinline__ void chunk_store_div(T* orow, const float (&ev)[VPT][Vec<T>::N],
                                                uint32_t j0, uint32_t jstep, uint32_t jhi,
                                                uint32_t len, float sum) {
    constexpr int V = Vec<T>::N;
    const RowDiv div(sum);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const uint32_t j = j0 + k * jstep;
        if (j < jhi) {
            float o[V];
            if (j * V + V <= len) {  // every key valid: RowDiv's paired fast path
                bool redo = div.ieee;
#pragma unroll
                for (int e = 0; e < V; e += 2) {
                    const float2 q = div.fast2(f2(ev[k][e], ev[k][e + 1]), redo);
                    o[e] = q.x;
                    o[e + 1] = q.y;
                }
                if (redo) {
#pragma unroll
                    for (int e = 0; e < V; ++e) o[e] = __fdiv_rn(ev[k][e], sum);
                }
            } else if (j * V < len) {  // the straddling vector: IEEE divide, 0 past len
#pragma unroll
                for (int e = 0; e < V; ++e) o[e] = j * V + e < len ? __fdiv_rn(ev[k][e], sum) : 0.0f;
            } else {
#pragma unroll
                for (int e = 0; e < V; ++e) o[e] = 0.0f;
            }
            st_stream(orow + (uint64_t)j * V, Vec<T>::pack(o));
        }
    }
}

// Vectors per thread: 32 row elements for bf16 (2 bytes each in flight), 16
// for f32, so the kept exp values fit the register budgets below.
constexpr int SMAX_VPT = 4;

// ---- rows read straight from HBM: tiles of rows, one CTA per row (BIG), or a
// cluster of CTAs per row --------------------------------------------------------
// cl == 1: a CTA holds blockDim / tpr rows (tpr threads each); BIG: one row
// per CTA of up to 512 threads (128-register budget); cl > 1: 256-thread CTAs
// of a cluster split one row.
template <typename T, int VPT, bool BIG, bool MASK>
__global__ void __launch_bounds__(BIG ? 512 : 256, BIG ? 1 : 3)
    smax_rows_kernel(const T* x, T* out, SmaxArgs p) {
    constexpr int V = Vec<T>::N;
    __shared__ float red[32];
    __shared__ float cl_slot[2];
    const uint32_t nvec = p.cols / V;
    uint32_t vlo = 0, vhi = nvec;
    int rpc = 1, sub = 0, t = threadIdx.x;
    if (p.cl > 1) {
        const int rank = (int)cg::this_cluster().block_rank();
        const uint32_t per = (nvec + p.cl - 1) / p.cl;
        vlo = rank * per;
        vhi = min(nvec, vlo + per);
    } else {
        rpc = blockDim.x / p.tpr;
        sub = threadIdx.x / p.tpr;
        t = threadIdx.x % p.tpr;
    }
    for (uint64_t row0 = (uint64_t)(blockIdx.x / p.cl) * rpc; row0 < p.rows;
         row0 += (uint64_t)(gridDim.x / p.cl) * rpc) {
        const uint64_t row = row0 + sub;
        const bool active = row < p.rows;
        const uint32_t len = active ? valid_len(p, row) : 0;
        const uint32_t jhi = active ? vhi : 0;
        const T* xr = x + row * p.cols;
        const uint32_t j0 = vlo + t;
        uint4 raw[VPT];
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const uint32_t j = j0 + k * p.tpr;
            if (j < jhi && j * V < len) raw[k] = ld_stream(xr + (uint64_t)j * V);
        }
        float m = group_reduce(chunk_max<T, VPT, MASK>(raw, p, j0, p.tpr, jhi, len), red, p.tpr,
                               OpMaxF());
        if (p.cl > 1) {
            cg::cluster_group cluster = cg::this_cluster();
            if (threadIdx.x == 0) cl_slot[0] = m;
            cluster.sync();
            float mm = -INFINITY;
            for (int q = 0; q < p.cl; ++q) mm = fmaxf(mm, *cluster.map_shared_rank(&cl_slot[0], q));
            m = mm;
        }
        float ev[VPT][V];
        float sum = group_reduce(chunk_exp<T, VPT, MASK>(raw, ev, p, j0, p.tpr, jhi, len, m), red,
                                 p.tpr, OpAddF());
        if (p.cl > 1) {
            cg::cluster_group cluster = cg::this_cluster();
            if (threadIdx.x == 0) cl_slot[1] = sum;
            cluster.sync();
            float tot = 0.0f;
            for (int q = 0; q < p.cl; ++q) tot = fadd(tot, *cluster.map_shared_rank(&cl_slot[1], q));
            sum = tot;
            cluster.sync();  // peers finished reading this CTA's slots
        }
        chunk_store_div<T, VPT>(out + row * p.cols, ev, j0, p.tpr, jhi, len, sum);
    }
}

// ---- fallbacks -----------------------------------------------------------------
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
        const RowDiv div(sum);
        for (uint32_t j = threadIdx.x; j < p.cols; j += blockDim.x) {
            float o = 0.0f;
            if (j < len) o = div(expf(fsub(score(p, Vec<T>::load1(xr + j), j), m)));
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
        const RowDiv div(sum);
        for (uint64_t d = 0; d < dim; ++d)
            Vec<T>::store1(out + base + d * inner,
                           div(expf(fsub(Vec<T>::load1(x + base + d * inner), m))));
    }
}

// ---- launchers -------------------------------------------------------------------
static cudaError_t launch_cluster(const void* kern, void** args, SmaxArgs& p, cudaStream_t st) {
    const uint64_t cap = (uint64_t)1 << 30;
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
    return cudaLaunchKernelExC(&cfg, kern, args);
}

template <typename T, int VPT, bool MASK>
static cudaError_t launch_tiled(const T* x, T* out, SmaxArgs p, cudaStream_t st) {
    // One tile of 256 / tpr rows per 256-thread CTA; the hardware keeps the
    // next CTAs' loads in flight while resident ones compute.
    const int rpc = 256 / p.tpr;
    const uint64_t tiles = (p.rows + rpc - 1) / rpc, cap = (uint64_t)1 << 30;
    smax_rows_kernel<T, VPT, false, MASK>
        <<<(unsigned)(tiles < cap ? tiles : cap), 256, 0, st>>>(x, out, p);
    return cudaSuccess;
}

template <typename T, bool BIG, bool MASK>
static cudaError_t launch_long(const T* x, T* out, SmaxArgs p, cudaStream_t st) {
    auto kern = smax_rows_kernel<T, SMAX_VPT, BIG, MASK>;
    if (p.cl > 1) {
        void* args[] = {(void*)&x, (void*)&out, (void*)&p};
        return launch_cluster(reinterpret_cast<const void*>(kern), args, p, st);
    }
    const uint64_t cap = (uint64_t)1 << 30;
    kern<<<(unsigned)(p.rows < cap ? p.rows : cap), p.tpr, 0, st>>>(x, out, p);
    return cudaSuccess;
}

template <typename T, bool MASK>
static cudaError_t launch_vec(const T* x, T* out, SmaxArgs p, int vpt, bool tiled, bool big,
                              cudaStream_t st) {
    if (!tiled) return big ? launch_long<T, true, MASK>(x, out, p, st)
                           : launch_long<T, false, MASK>(x, out, p, st);
    if (vpt == 1) return launch_tiled<T, 1, MASK>(x, out, p, st);
    if (vpt == 2) return launch_tiled<T, 2, MASK>(x, out, p, st);
    return launch_tiled<T, SMAX_VPT, MASK>(x, out, p, st);
}

// ---- bf16 rows of up to 32 * 8 * VPT keys, no additive mask ---------------------
// One warp per row, lane l owning the 8-key vectors l, l + 32, ...; rows are
// taken in a grid-stride loop by a persistent grid.  Only vectors holding a
// valid key are read.  The output is bf16, so the f32 intermediate only has to
// be accurate far below half a bf16 ulp (2^-9 relative) for every output to
// be within one bf16 ulp of the reference; that allows:
//   * the row max taken on the packed bf16 keys (max.bf16x2): for scale > 0,
//     x -> RN(x * scale) is non-decreasing, so RN(max(x) * scale) is the max
//     of the scaled scores; NaN keys are skipped like f32::max skips them;
//   * exp(s - m) as ex2(x * (scale * log2 e) - m * log2 e): one paired FMA and
//     one ex2.approx (relative error ~2^-22, subnormal results kept) per key,
//     error ~|s - m| * 2^-24 relative, at most ~1e-5 for |s - m| <= 100;
//   * p = e / sum as ex2(x * (scale * log2 e) - m * log2 e - log2(sum)): the
//     exponent is recomputed in the store pass instead of keeping e, so a lane
//     holds only its packed keys (64 registers, 4 CTAs of 256 threads per SM:
//     measured 10% faster than keeping e at 2 CTAs per SM); lg2.approx adds
//     ~2^-22 absolute to the exponent, ~1.7e-7 relative to p.
__device__ __forceinline__ float ex2_approx(float t) {
    float y;
    asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(t));
    return y;
}
__device__ __forceinline__ float lg2_approx(float t) {
    float y;
    asm("lg2.approx.f32 %0, %1;" : "=f"(y) : "f"(t));
    return y;
}
__device__ __forceinline__ uint32_t bf16x2_max(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("max.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
// Keys k >= keep (0 < keep < 8) of a vector of 8 bf16 set to `fill`.
__device__ __forceinline__ uint4 bf16_tail(uint4 v, uint32_t keep, uint32_t fill) {
    uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if (2u * i >= keep) w[i] = fill | (fill << 16);
        else if (2u * i + 1 >= keep) w[i] = (w[i] & 0xffffu) | (fill << 16);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

constexpr float kLog2e = 1.4426950408889634f;

template <int VPT>
__global__ void __launch_bounds__(256, 4)
    smax_bf16_warp_kernel(const bf16_t* __restrict__ x, bf16_t* __restrict__ out, SmaxArgs p) {
    const uint32_t lane = threadIdx.x & 31u;
    const uint64_t warp0 = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const uint64_t nwarps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
    const uint32_t nvec = p.cols >> 3;
    const float c1 = fmul(p.scale, kLog2e);
    for (uint64_t row = warp0; row < p.rows; row += nwarps) {
        const uint32_t len = valid_len(p, row);
        const uint32_t nv = (len + 7u) >> 3;  // vectors holding a valid key
        const uint32_t tail = len & 7u;       // valid keys of vector nv - 1 (0: all 8)
        const uint4* xr = reinterpret_cast<const uint4*>(x + row * p.cols);
        uint4* orow = reinterpret_cast<uint4*>(out + row * p.cols);
        uint4 raw[VPT];
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const uint32_t v = lane + 32u * k;
            if (v < nv) raw[k] = ld_stream(xr + v);
        }
        uint32_t mx = 0xff80ff80u;  // (-inf, -inf)
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const uint32_t v = lane + 32u * k;
            if (v < nv) {
                if (tail && v == nv - 1) raw[k] = bf16_tail(raw[k], tail, 0xff80u);
                mx = bf16x2_max(mx, bf16x2_max(bf16x2_max(raw[k].x, raw[k].y),
                                               bf16x2_max(raw[k].z, raw[k].w)));
            }
        }
        const float m = warp_max(fmaxf(bf16_lo(mx), bf16_hi(mx)));
        const float c2 = fmul(-fmul(m, p.scale), kLog2e);
        float2 acc = f2(0.0f, 0.0f);
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const uint32_t v = lane + 32u * k;
            if (v < nv) {
                const uint32_t w[4] = {raw[k].x, raw[k].y, raw[k].z, raw[k].w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float2 t = __ffma2_rn(f2(bf16_lo(w[i]), bf16_hi(w[i])), f2(c1, c1), f2(c2, c2));
                    acc = fadd2(acc, f2(ex2_approx(t.x), ex2_approx(t.y)));
                }
            }
        }
        const float c3 = fsub(c2, lg2_approx(warp_sum(fadd(acc.x, acc.y))));
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const uint32_t v = lane + 32u * k;
            if (v < nvec) {
                uint4 o = make_uint4(0u, 0u, 0u, 0u);
                if (v < nv) {
                    const uint32_t r[4] = {raw[k].x, raw[k].y, raw[k].z, raw[k].w};
                    uint32_t w[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float2 t = __ffma2_rn(f2(bf16_lo(r[i]), bf16_hi(r[i])), f2(c1, c1), f2(c3, c3));
                        w[i] = pack_bf16x2(ex2_approx(t.x), ex2_approx(t.y));
                    }
                    o = make_uint4(w[0], w[1], w[2], w[3]);
                    if (tail && v == nv - 1) o = bf16_tail(o, tail, 0u);
                }
                st_stream(orow + v, o);
            }
        }
    }
}

template <int VPT>
static cudaError_t launch_bf16_warp(const bf16_t* x, bf16_t* out, const SmaxArgs& p, cudaStream_t st) {
    const auto kern = smax_bf16_warp_kernel<VPT>;
    const uint64_t want = (p.rows + 7) / 8;
    // two CTAs per resident slot: measured ~2% faster than one
    const uint64_t cap = 2ull * resident_blocks(reinterpret_cast<const void*>(kern), 256, 0) * sm_count();
    const unsigned grid = (unsigned)(want < cap ? want : cap);
    kern<<<grid, 256, 0, st>>>(x, out, p);
    return cudaSuccess;
}

// The bf16 warp kernel serves rows of whole vectors up to 2048 keys when the
// scores are x * scale with 0 < scale < inf and no additive mask.
template <typename T>
static bool try_bf16_warp(const T* x, T* out, const SmaxArgs& p, cudaStream_t st, cudaError_t& e) {
    if constexpr (!std::is_same<T, bf16_t>::value) {
        return false;
    } else {
        if (p.mask || !(p.scale > 0.0f && p.scale <= 3.4028235e38f)) return false;
        if (p.cols % 8 != 0 || p.cols > 2048 || !aligned16(x) || !aligned16(out)) return false;
        const uint32_t nvec = p.cols / 8;
        if (nvec <= 32) e = launch_bf16_warp<1>(x, out, p, st);
        else if (nvec <= 64) e = launch_bf16_warp<2>(x, out, p, st);
        else if (nvec <= 128) e = launch_bf16_warp<4>(x, out, p, st);
        else e = launch_bf16_warp<8>(x, out, p, st);
        return true;
    }
}

template <typename T>
static int rows_dispatch(const char* name, const T* x, T* out, SmaxArgs p, cudaStream_t st) {
    constexpr int V = Vec<T>::N;
    // 32-bit multiply-shift divisions for the per-row lens / causal lookups.
    p.narrow = p.rows < 0xffffffffull;
    p.len_div = FastDiv((uint32_t)(p.rows_per_len < 0xffffffffull ? p.rows_per_len : 0xffffffffull));
    p.causal_div = FastDiv((uint32_t)(p.causal_q ? p.causal_q : 1));
    {
        cudaError_t e = cudaSuccess;
        if (try_bf16_warp(x, out, p, st, e)) {
            if (e != cudaSuccess) {
                cudaGetLastError();
                return set_error(OXIDE_ERR_LAUNCH, "%s: launch failed: %s", name, cudaGetErrorString(e));
            }
            return check_launch(name);
        }
    }
    constexpr int VT = SMAX_VPT;
    const uint64_t cap = (uint64_t)1 << 30;
    const uint64_t nvec = p.cols / V;
    const bool vec = p.cols % V == 0 && aligned16(x) && aligned16(out);
    int vpt = 0;
    bool tiled = false, big = false;
    p.cl = 1;
    if (vec && nvec <= 32ull * VT) {  // a warp per row, 8 rows per tile
        p.tpr = 32;
        vpt = 1;
        while ((uint64_t)vpt * 32 < nvec) vpt *= 2;
        tiled = true;
    } else if (vec && nvec <= 256ull * VT) {  // 64..256 threads per row
        uint64_t tpr = 64;
        while (tpr * VT < nvec) tpr *= 2;
        p.tpr = (int)tpr;
        vpt = VT;
        tiled = true;
    } else if (vec && nvec <= 512ull * VT && p.rows >= 2ull * sm_count()) {
        p.tpr = (int)(((nvec + VT - 1) / VT + 31) / 32 * 32);  // one CTA per row
        vpt = VT;
        big = true;
    } else if (vec && nvec <= 8ull * 256 * VT) {
        p.tpr = 256;  // a cluster of up to 8 CTAs per row
        const uint64_t cl = (nvec + 256ull * VT - 1) / (256ull * VT);
        int c2 = 1;
        while ((uint64_t)c2 < cl) c2 *= 2;
        p.cl = c2;
        vpt = VT;
    }
    cudaError_t e = cudaSuccess;
    if (vpt == 0) {
        smax_rows_scalar_kernel<T><<<(unsigned)(p.rows < cap ? p.rows : cap), 256, 0, st>>>(x, out, p);
    } else if (p.mask) {
        e = launch_vec<T, true>(x, out, p, vpt, tiled, big, st);
    } else {
        e = launch_vec<T, false>(x, out, p, vpt, tiled, big, st);
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
